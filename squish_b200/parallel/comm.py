"""Tensor-parallel collectives for one process per GPU.

Two implementations behind one interface:

  * ``nvlink`` (default on GPUs): buffers shared by CUDA IPC across the group. Decode-sized
    row-parallel outputs (<= 256 tokens) run the GEMM into a local scratch and then one
    one-shot all-reduce kernel (``tp_oneshot``: each CTA publishes its chunk in a
    double-buffered peer-visible slot, waits for the peers' chunk, sums in rank order);
    larger ones push output tiles into every rank's receive buffer from the GEMM epilogue and
    ``tp_reduce`` sums them (csrc/comm.cu). The vocab-parallel logits are gathered with P2P
    stores. No NCCL call on the step's hot path.
  * ``sp`` (sequence parallel): rank r owns a contiguous block of the step's token rows; the
    row-parallel GEMMs (o_proj, down_proj) route each partial row to its owner from the GEMM
    epilogue (reduce-scatter: (tp-1)/tp of the rows cross NVLink, not (tp-1) copies of all of
    them), one kernel per layer half sums the partials into the owned residual rows, applies
    the next RMSNorm and pushes the normalised rows to every rank (all-gather), and the
    column-parallel GEMM (qkv, gate_up) waits for the gather inside its activation producer
    while its weights already stream; MoE layers replace the FFN's all-gather / reduce-scatter
    with the expert-parallel all-to-all (``setup_ep`` / ``ep_dispatch`` / ``ep_combine``,
    csrc/ep_a2a.cu): each owned row goes only to the ranks holding its routed experts and the
    weighted expert sums come back through the reduce-scatter blocks;
  * ``nccl``: the same math with torch.distributed all_reduce / all_gather (the baseline;
    also what CPU ranks use, over gloo).

Every rank runs the same sequence of collectives in the same order (the engine's host
logic is replicated SPMD on every rank), which both protocols rely on.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .._ext import native
from .shard import vocab_shard


ONESHOT_MAX_CTAS = 148  # csrc/comm.h kOneshotMaxCtas
# Row-parallel outputs of at most this many tokens take the one-shot all-reduce (GEMM into a
# local scratch, then one kernel that publishes, waits and sums); larger ones the fused
# push-from-the-epilogue path
ONESHOT_MAX_TOKENS = int(os.environ.get("SQ_TP_ONESHOT_MAX_TOKENS", "256"))


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
        self.link_bytes = 0  # host-side tally of collective payload bytes received by this rank
        v0, v1 = vocab_shard(vocab, self.rank, self.tp)
        self.v0, self.v1 = v0, v1
        self.per = vocab_shard(vocab, 0, self.tp)[1]  # padded shard width (ranks' shards all fit in it)
        self._ipc = []
        if mode in ("nvlink", "sp"):
            self._check_peer_access()
            self._setup_peer()
            if mode == "sp":
                self._setup_sp()
        else:
            self.tmp = torch.empty(max_tokens, hidden, dtype=torch.bfloat16 if mode == "nccl" else torch.float32,
                                   device=self.device)
            self.logits_full = torch.empty(max_rows, vocab, dtype=self.tmp.dtype, device=self.device)
            self.gath = torch.empty(self.tp * max_rows * self.per, dtype=self.tmp.dtype, device=self.device)

    # ------------------------------------------------------------------ NVLink peer memory
    def _check_peer_access(self) -> None:
        """Every rank must reach every peer's memory directly (NVLink / NVSwitch peer access);
        all ranks agree before any IPC buffer is opened."""
        n = torch.cuda.device_count()
        me = self.device.index
        ok = all(torch.cuda.can_device_access_peer(me, j) for j in range(n) if j != me) if n > 1 else True
        flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, group=self.group)
        if int(flag.item()):
            raise RuntimeError(f"tp_mode '{self.mode}' needs peer access between every pair of GPUs "
                               "(NVLink / NVSwitch); use tp_mode 'nccl'")


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
        # one-shot all-reduce: double-buffered partial slots and per-chunk arrival flags
        os_part = self._alloc_shared(2 * T * H * 2)
        os_flags = self._alloc_shared(ONESHOT_MAX_CTAS * tp * 4)
        self.os_part_ptrs = torch.tensor(os_part, **i64)
        self.os_flag_ptrs = torch.tensor(os_flags, **i64)
        self.os_tmp = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        self.os_seq = torch.zeros(1, dtype=torch.int32, device=dev)
        self.os_done = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ sequence parallel
    def _setup_sp(self):
        """Buffers of the sequence-parallel collectives: a reduce-scatter receive area
        [tp source][rows per rank][H], the all-gather buffer [T][H] that the next GEMM reads,
        and counters (reduce-scatter [2 parity][tp], all-gather [tp]) -- all in IPC memory
        that the peers store into."""
        tp, T, H = self.tp, self.max_tokens, self.hidden
        dev = self.device
        R = -(-T // tp)
        self.sp_rows_max = R
        recv = self._alloc_shared(tp * R * H * 2)
        xg = self._alloc_shared(T * H * 2)
        flags = self._alloc_shared(3 * tp * 4)
        i64 = dict(dtype=torch.int64, device=dev)
        self.sp_push_dst = torch.tensor([p + 2 * self.rank * R * H for p in recv], **i64)
        self.sp_push_flags = torch.tensor([p + 4 * self.rank for p in flags], **i64)
        self.sp_ag_dst = torch.tensor(xg, **i64)
        self.sp_ag_flag_ptrs = torch.tensor([p + 4 * (2 * tp + self.rank) for p in flags], **i64)
        idx = dev.index
        self.sp_recv = native().tensor_from_ptr(recv[self.rank], [tp * R * H], torch.bfloat16, idx)
        self.xg = native().tensor_from_ptr(xg[self.rank], [T, H], torch.bfloat16, idx)
        fl = native().tensor_from_ptr(flags[self.rank], [3 * tp], torch.int32, idx)
        self.sp_rs_flags, self.sp_ag_flags = fl[: 2 * tp], fl[2 * tp:]
        self.sp_seq = torch.zeros(1, dtype=torch.int32, device=dev)
        self.sp_done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.sp_ag_done = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    # ------------------------------------------------------------------ expert-parallel all-to-all
    def setup_ep(self, top_k: int, experts_local: int) -> None:
        """Receive slots of the expert-parallel all-to-all (sequence-parallel mode; csrc/ep_a2a.cu):
        per source rank, R rows of x and R x K (local expert id | -1, routing weight) pairs, and one
        dispatch counter per source -- IPC memory that the sources store into. The combine goes
        back through the reduce-scatter buffers above."""
        if self.mode != "sp":
            raise ValueError("the expert-parallel all-to-all runs in the sequence-parallel mode")
        if getattr(self, "ep_k", None) == top_k and self.ep_experts == experts_local:
            return
        tp, R, H, K = self.tp, self.sp_rows_max, self.hidden, top_k
        x = self._alloc_shared(tp * R * H * 2)
        ids = self._alloc_shared(tp * R * K * 4)
        w = self._alloc_shared(tp * R * K * 4)
        fl = self._alloc_shared(tp * 4)
        i64 = dict(dtype=torch.int64, device=self.device)
        idx = self.device.index
        self.ep_k, self.ep_experts = K, experts_local
        self.ep_x_ptrs = torch.tensor(x, **i64)
        self.ep_ids_ptrs = torch.tensor(ids, **i64)
        self.ep_w_ptrs = torch.tensor(w, **i64)
        self.ep_flag_ptrs = torch.tensor([p + 4 * self.rank for p in fl], **i64)
        self.ep_x = native().tensor_from_ptr(x[self.rank], [tp * R, H], torch.bfloat16, idx)
        self.ep_ids = native().tensor_from_ptr(ids[self.rank], [tp * R * K], torch.int32, idx)
        self.ep_w = native().tensor_from_ptr(w[self.rank], [tp * R * K], torch.float32, idx)
        self.ep_flags = native().tensor_from_ptr(fl[self.rank], [tp], torch.int32, idx)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def ep_own(self, T: int) -> tuple[int, int]:
        """(first owned row, owned rows) of this rank in a T-token step."""
        R = self.sp_rows(T)
        r0 = self.rank * R
        return r0, max(0, min(R, T - r0))

    def ep_dispatch(self, x_own: torch.Tensor, logits: torch.Tensor | None, renorm: bool, ids: torch.Tensor,
                    w: torch.Tensor, T: int) -> None:
        """Route each owned row (x_own [own, H]; router logits [own, E], or None when ids / w
        already hold the [own, K] global expert ids and weights) and send it to the ranks
        holding its experts. The receivers' arrival wait runs in ``ep_align``."""
        from ..ops import kernels as K_

        R = self.sp_rows(T)
        own = x_own.shape[0]
        if T > self.max_tokens:
            raise ValueError("expert-parallel step exceeds the sequence-parallel buffers")
        native().ep_dispatch(x_own, logits, bool(renorm), ids, w, own, R, self.ep_k, self.ep_experts, self.rank,
                             self.tp, self.ep_x_ptrs, self.ep_ids_ptrs, self.ep_w_ptrs, self.ep_flag_ptrs)
        K_._count()

    def ep_align(self, T: int, bn: int, sorted_slot, slot_pos, tile_expert, num_tiles, counts) -> None:
        """Wait (bounded) for every source's R dispatched row slots of this step, then lay the
        received slots out expert-sorted for the grouped GEMMs (one kernel)."""
        from ..ops import kernels as K_

        R = self.sp_rows(T)
        TK = self.tp * R * self.ep_k
        K_.moe_align(self.ep_ids[:TK], self.ep_experts, bn, sorted_slot, slot_pos, tile_expert, num_tiles, counts,
                     wait_flags=self.ep_flags, wait_expect=R, status=self.status)

    def ep_combine(self, ys: torch.Tensor, slot_pos: torch.Tensor, T: int) -> int:
        """Weighted expert outputs of the received rows back to their owners' reduce-scatter
        blocks; returns the arrivals each owner expects per source (for rs_norm_ag)."""
        from ..ops import kernels as K_

        R = self.sp_rows(T)
        # link bytes: dispatch (at most every owned row to every peer) + combine rows
        self.link_bytes += 2 * (self.tp - 1) * R * self.hidden * 2
        native().ep_combine(ys, slot_pos, self.ep_w, R, self.ep_k, self.tp, T, self.sp_push_dst, self.hidden,
                            self.sp_push_flags, self.tp, self.sp_seq)
        K_._count()
        return R

    def sp_rows(self, T: int) -> int:
        """Token rows each rank owns in a T-token step (the last rank may own fewer or none)."""
        return -(-T // self.tp)

    def ag_expect(self, T: int) -> int:
        return self.sp_rows(T)  # CTAs of each source's tp_rs_norm_ag (one per owned row)

    def gemm_rs(self, x: torch.Tensor, w, ws) -> int:
        """Row-parallel GEMM whose partial rows go to their owner ranks (reduce-scatter routing
        in the GEMM epilogue). Returns the launch's CTA count, the owners' expected arrivals."""
        from ..ops import kernels as K

        T = x.shape[0]
        if T > self.max_tokens or w.n != self.hidden:
            raise ValueError("row-parallel output exceeds the sequence-parallel buffers")
        e = native().w4a16_gemm_rs(x, w.wq, w.n, w.k, w.group, w.n, self.sp_push_dst, self.sp_push_flags, self.tp,
                                   self.sp_seq, self.tp, self.sp_rows(T), ws.gemm_ws, ws.gemm_counters, ws.status)
        K._count()
        return int(e)

    def rs_norm_ag(self, h: torch.Tensor, norm_w: torch.Tensor, eps: float, T: int, rs_expect: int,
                   local_only: bool = False) -> None:
        """Owned rows: h += sum of the tp partials; then RMSNorm(h) into every rank's xg (only
        this rank's xg with local_only: the input of an expert-parallel dispatch)."""
        from ..ops import kernels as K

        R = self.sp_rows(T)
        self.link_bytes += (1 if local_only else 2) * (self.tp - 1) * R * self.hidden * 2  # RS in (+ AG in)
        native().tp_rs_norm_ag(self.sp_recv, self.sp_rows_max * self.hidden, self.hidden, self.sp_rs_flags,
                               int(rs_expect), h, norm_w, float(eps), self.sp_ag_dst, self.hidden,
                               self.sp_ag_flag_ptrs, self.rank, self.tp, R, T, self.sp_seq, self.sp_done,
                               self.status, bool(local_only))
        K._count()

    def ag_wait(self, T: int) -> None:
        from ..ops import kernels as K

        native().tp_ag_wait(self.sp_ag_flags, self.ag_expect(T), self.tp, self.status)
        K._count()

    def gemm_ag(self, w, out: torch.Tensor, T: int, silu_mul: bool, ws) -> torch.Tensor:
        """Column-parallel GEMM over the all-gathered rows xg[:T]: the INT4 decode kernel waits
        for the gather inside its activation producer (the weights stream meanwhile); the
        bf16 prefill path and rotated weights wait in a separate one-CTA kernel first."""
        from ..ops import kernels as K

        x = self.xg[:T]
        if T >= K.DQ_GEMM_MIN_M or w.rot is not None or w.lr_a is not None:
            self.ag_wait(T)
            return K.w4a16_linear(x, w, out=out, silu_mul=silu_mul, ws=ws)
        native().w4a16_gemm(x, w.wq, w.sz, w.n, w.k, w.group, out, w.bias, None,
                            K.EPI_SILU_MUL if silu_mul else K.EPI_PLAIN, ws.gemm_ws, ws.gemm_counters, ws.status,
                            None, w.fmt, w.codebook, ag_flags=self.sp_ag_flags, ag_done=self.sp_ag_done,
                            ag_expect=self.ag_expect(T), ag_tp=self.tp)
        K._count()
        return out

    # ------------------------------------------------------------------ collectives
    def gemm_allreduce(self, x: torch.Tensor, w, h: torch.Tensor, ws) -> None:
        """h += all_reduce(x @ w^T) over the group (w: this rank's row-parallel shard)."""
        from ..ops import kernels as K

        T = x.shape[0]
        self.link_bytes += (self.tp - 1) * T * h.shape[1] * 2  # peers' partials received by this rank
        if self.mode not in ("nvlink", "sp"):
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
        if T <= ONESHOT_MAX_TOKENS:
            part = K.w4a16_linear(x, w, out=self.os_tmp[:T], ws=ws)
            native().tp_oneshot(part, self.os_part_ptrs, self.max_tokens * self.hidden, self.os_flag_ptrs, h, True,
                                self.rank, self.tp, self.os_seq, self.os_done, self.status)
            K._count()
            return
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
        if self.mode not in ("nvlink", "sp"):
            tmp = self.tmp[:T]
            tmp.copy_(x.to(tmp.dtype))
            dist.all_reduce(tmp, group=self.group)
            h.add_(tmp.to(h.dtype))
            return
        if T > self.max_tokens or x.shape[1] != self.hidden:
            raise ValueError("all-reduce input exceeds the peer buffers")
        self.link_bytes += (self.tp - 1) * T * self.hidden * 2
        if T <= ONESHOT_MAX_TOKENS and x.dtype == torch.bfloat16 and x.stride(1) == 1:
            native().tp_oneshot(x, self.os_part_ptrs, self.max_tokens * self.hidden, self.os_flag_ptrs, h, True,
                                self.rank, self.tp, self.os_seq, self.os_done, self.status)
            K._count()
            return
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

        if self.mode not in ("nvlink", "sp"):
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
        if self.mode in ("nvlink", "sp"):
            s = int(self.status.item())
            if s:
                raise RuntimeError(f"tensor-parallel collective failed (status {s}: a peer did not arrive in time)")

    def close(self) -> None:
        if self.mode not in ("nvlink", "sp"):
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
