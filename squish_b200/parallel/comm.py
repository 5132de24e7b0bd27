"""Tensor-parallel collectives for one process per GPU.

Two implementations behind one interface:

  * ``nvlink`` (default on GPUs): buffers shared by CUDA IPC across the group; the
    row-parallel GEMM pushes its output tiles into every rank's receive buffer from the
    GEMM epilogue and ``tp_reduce`` sums them (csrc/comm.cu); the vocab-parallel logits are
    gathered with P2P stores. No NCCL call on the step's hot path.
  * ``nccl``: the same math with torch.distributed all_reduce / all_gather (the baseline;
    also what CPU ranks use, over gloo).

Every rank runs the same sequence of collectives in the same order (the engine's host
logic is replicated SPMD on every rank), which both protocols rely on.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._ext import native
from .shard import vocab_shard


class TPComm:
    def __init__(self, mode: str, max_tokens: int, hidden: int, max_rows: int, vocab: int, group=None,
                 device: torch.device | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.tp = dist.get_world_size(group)
        self.mode = mode
        self.device = device or (torch.device("cuda", torch.cuda.current_device()) if mode != "cpu"
                                 else torch.device("cpu"))
        self.max_tokens, self.hidden, self.max_rows, self.vocab = max_tokens, hidden, max_rows, vocab
        v0, v1 = vocab_shard(vocab, self.rank, self.tp)
        self.v0, self.v1 = v0, v1
        self.per = vocab_shard(vocab, 0, self.tp)[1]  # padded shard width (ranks' shards all fit in it)
        self._ipc = []
        if mode == "nvlink":
            self._setup_peer()
        else:
            self.tmp = torch.empty(max_tokens, hidden, dtype=torch.bfloat16 if mode == "nccl" else torch.float32,
                                   device=self.device)
            self.logits_full = torch.empty(max_rows, vocab, dtype=self.tmp.dtype, device=self.device)
            self.gath = torch.empty(self.tp * max_rows * self.per, dtype=self.tmp.dtype, device=self.device)

    # ------------------------------------------------------------------ NVLink peer memory
    def _alloc_shared(self, nbytes: int) -> list[int]:
        """One IPC buffer per rank; returns every rank's device pointer (own first opened)."""
        ptr, handle = native().ipc_alloc(int(nbytes))
        own = int(ptr.item())
        self._ipc.append(("free", own))
        hs = [None] * self.tp
        dist.all_gather_object(hs, handle.numpy().tobytes(), group=self.group)
        ptrs = []
        for r, h in enumerate(hs):
            if r == self.rank:
                ptrs.append(own)
            else:
                p = native().ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8))
                self._ipc.append(("close", p))
                ptrs.append(p)
        return ptrs

    def _setup_peer(self):
        tp, T, H = self.tp, self.max_tokens, self.hidden
        dev = self.device
        self.src_stride = T * H                           # elements per source slot
        self.recv_stride = tp * self.src_stride           # elements per parity
        self.max_tiles = (H // 128 + 2) * (T // 16 + 2)
        nflag_reduce = 2 * tp * self.max_tiles
        nflag = nflag_reduce + 2 * tp
        recv = self._alloc_shared(2 * self.recv_stride * 2)
        flags = self._alloc_shared(nflag * 4)
        logits = self._alloc_shared(self.max_rows * self.vocab * 2)
        i64 = dict(dtype=torch.int64, device=dev)
        self.push_dst = torch.tensor([p + 2 * self.rank * self.src_stride for p in recv], **i64)
        self.push_flags = torch.tensor([p + 4 * self.rank * self.max_tiles for p in flags], **i64)
        self.gather_dst = torch.tensor(logits, **i64)
        self.gather_flags = torch.tensor([p + 4 * nflag_reduce for p in flags], **i64)
        idx = dev.index
        self.recv = native().tensor_from_ptr(recv[self.rank], [2 * self.recv_stride], torch.bfloat16, idx)
        self.flags = native().tensor_from_ptr(flags[self.rank], [nflag], torch.int32, idx)
        self.flags_gather = self.flags[nflag_reduce:]
        self.logits_full = native().tensor_from_ptr(logits[self.rank], [self.max_rows, self.vocab], torch.bfloat16,
                                                    idx)
        self.seq = torch.zeros(1, dtype=torch.int32, device=dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ collectives
    def gemm_allreduce(self, x: torch.Tensor, w, h: torch.Tensor, ws) -> None:
        """h += all_reduce(x @ w^T) over the group (w: this rank's row-parallel shard)."""
        from ..ops import kernels as K

        T = x.shape[0]
        if self.mode != "nvlink":
            tmp = self.tmp[:T]
            if self.mode == "cpu":
                tmp.copy_(x.float() @ w.T)
            else:
                K.w4a16_linear(x, w, out=tmp, ws=ws)
            dist.all_reduce(tmp, group=self.group)
            h.add_(tmp.to(h.dtype))
            return
        N = w.n
        if T > self.max_tokens or N != self.hidden:
            raise ValueError("row-parallel output exceeds the peer buffers")
        bn, nt, _, _, _ = native().gemm_plan(T, N, w.k)
        if ((N + 128 * nt - 1) // (128 * nt)) * ((T + bn - 1) // bn) > self.max_tiles:
            raise ValueError("GEMM tile grid exceeds the flag array")
        bn, nt, splits, gx, gy = native().w4a16_gemm_push(
            x, w.wq, N, w.k, w.group, N, self.push_dst, self.push_flags, self.recv_stride,
            self.tp * self.max_tiles, self.seq, self.tp, ws.gemm_ws, ws.gemm_counters, ws.status)
        native().tp_reduce(self.recv, self.recv_stride, self.src_stride, N, self.flags, self.tp * self.max_tiles,
                           self.max_tiles, splits, h, True, T, N, bn, 128 * nt, gx, gy, self.tp, self.seq,
                           self.done, self.status)
        K._count(2)

    def allreduce_add(self, x: torch.Tensor, h: torch.Tensor) -> None:
        """h += all_reduce(x) over the group (x: [T, hidden] partial, e.g. local experts' output)."""
        from ..ops import kernels as K

        T = x.shape[0]
        if self.mode != "nvlink":
            tmp = self.tmp[:T]
            tmp.copy_(x.to(tmp.dtype))
            dist.all_reduce(tmp, group=self.group)
            h.add_(tmp.to(h.dtype))
            return
        if T > self.max_tokens or x.shape[1] != self.hidden:
            raise ValueError("all-reduce input exceeds the peer buffers")
        N, tile_m = x.shape[1], 64
        gx, gy = (N + 127) // 128, (T + tile_m - 1) // tile_m
        if gx * gy > self.max_tiles:
            raise ValueError("all-reduce tile grid exceeds the flag array")
        native().tp_push(x, self.push_dst, self.recv_stride, N, self.push_flags, self.tp * self.max_tiles, tile_m,
                         gx, gy, self.tp, self.seq)
        native().tp_reduce(self.recv, self.recv_stride, self.src_stride, N, self.flags, self.tp * self.max_tiles,
                           self.max_tiles, 1, h, True, T, N, tile_m, 128, gx, gy, self.tp, self.seq, self.done,
                           self.status)
        K._count(2)

    def gather_logits(self, local: torch.Tensor, B: int) -> torch.Tensor:
        """[B, v1 - v0] vocab shard on every rank -> [B, vocab] on every rank."""
        from ..ops import kernels as K

        if self.mode != "nvlink":
            pad = torch.zeros(B, self.per, dtype=self.gath.dtype, device=self.device)
            pad[:, : local.shape[1]] = local
            g = self.gath[: self.tp * B * self.per].view(self.tp * B, self.per)
            dist.all_gather_into_tensor(g, pad, group=self.group)
            full = g.view(self.tp, B, self.per).permute(1, 0, 2).reshape(B, self.tp * self.per)[:, : self.vocab]
            self.logits_full[:B].copy_(full)
            return self.logits_full[:B]
        native().tp_gather(local, self.gather_dst, self.vocab, 0, self.v0, self.gather_flags, self.flags_gather,
                           self.tp, 32, self.rank, self.tp, self.seq, self.status)
        K._count(2)
        return self.logits_full[:B]

    def check(self) -> None:
        if self.mode == "nvlink":
            s = int(self.status.item())
            if s:
                raise RuntimeError(f"tensor-parallel collective failed (status {s}: a peer did not arrive in time)")

    def close(self) -> None:
        if self.mode != "nvlink":
            return
        torch.cuda.synchronize(self.device)
        for kind, p in reversed(self._ipc):
            if kind == "close":
                native().ipc_close(p)
        dist.barrier(group=self.group)
        for kind, p in self._ipc:
            if kind == "free":
                native().ipc_free(p)
        self._ipc = []
