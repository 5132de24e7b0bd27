"""Tensor-parallel model runners: the single-GPU runner over this rank's shard, with the
row-parallel outputs all-reduced and the vocab-parallel logits gathered.

``TPCudaRunner``: o_proj and down_proj run as one fused GEMM+all-reduce over NVLink (or the
NCCL baseline), or, in the sequence-parallel mode, as GEMM->reduce-scatter with the RMSNorm
and all-gather fused into one kernel and the gather wait fused into the next GEMM (MoE layers:
the owned rows go to the ranks holding their experts and the expert sums come back through the
reduce-scatter blocks, an all-to-all over peer memory instead of an all-reduce); the LM
head computes this rank's vocabulary slice and the slices are
gathered into a full logits row on every rank, so every rank samples the same tokens and
the engine's host logic can run replicated on every rank. ``TorchTPRunner`` is the CPU
(gloo) counterpart used to test the sharding end to end.
"""
from __future__ import annotations

import torch

from ..models.decoder import CudaRunner, TorchPagedRunner
from ..models.weights import Checkpoint
from .comm import TPComm
from .shard import shard_checkpoint


class TPCudaRunner(CudaRunner):
    def __init__(self, ck: Checkpoint, device, num_pages: int, comm: TPComm, **kw):
        self.full_cfg = ck.config
        self.comm = comm
        local = shard_checkpoint(ck, comm.rank, comm.tp)
        super().__init__(local, device, num_pages, **kw)
        R = self.logits.shape[0]
        self.logits_local = torch.empty(R, comm.v1 - comm.v0, dtype=torch.bfloat16, device=self.device)
        del self.logits
        self.logits = comm.logits_full
        moe = [lw.moe for lw in self.layers if lw.moe is not None]
        if moe and comm.mode == "sp":
            # expert parallelism with the all-to-all: the MoE scratch covers every source's slots
            from ..models.moe import MoEScratch

            comm.setup_ep(self.cfg.num_experts_per_tok, self.cfg.num_local_experts or self.cfg.num_experts)
            self.moe_scratch = MoEScratch(self.cfg, comm.tp * comm.sp_rows_max, self.device)
            for mo in moe:
                mo.scratch = self.moe_scratch
        else:
            for mo in moe:  # expert parallelism: all-reduce the local experts' partial output
                mo.ep_reduce = lambda part, h: self.comm.allreduce_add(part, h)

    def forward(self, st, m):
        if self.comm.mode != "sp":
            return super().forward(st, m)
        return self._forward_sp(st, m)

    def _forward_sp(self, st, m):
        """Sequence-parallel step: the residual rows of the step are split over the ranks;
        o_proj / down_proj reduce-scatter their partial rows to the owners from the GEMM
        epilogue, one kernel per half layer adds them to the owned residual rows, applies the
        next RMSNorm and all-gathers the normalised rows, and qkv / gate_up read the gathered
        rows as soon as every rank has pushed its part."""
        from .. import ops

        cfg, comm, ws = self.cfg, self.comm, self.ws
        T, Bd = st.num_tokens, st.num_decode
        h = self.h[:T]
        torch.index_select(self.embed, 0, m["ids"], out=h)
        dsplit = ops.kernels.decode_splits(max(Bd, 1), cfg.num_kv_heads, max(st.max_decode_ctx, 1)) if Bd else (1, 1)
        xg = comm.xg[:T]
        ops.rmsnorm(h, self.layers[0].ln1, cfg.rms_eps, out=xg)  # every row is valid everywhere at the start
        L = len(self.layers)
        for li, lw in enumerate(self.layers):
            if li == 0:
                qkv = ops.w4a16_linear(xg, lw.qkv, out=self.qkv[:T], ws=ws)
            else:
                qkv = comm.gemm_ag(lw.qkv, self.qkv[:T], T, False, ws)
            attn = self._attention(li, lw, qkv, st, m, dsplit)
            e = comm.gemm_rs(attn, lw.o, ws)
            if lw.moe is not None:  # owned rows normalised locally, then the expert all-to-all
                comm.rs_norm_ag(h, lw.ln2, cfg.rms_eps, T, e, local_only=True)
                r0, own = comm.ep_own(T)
                e = lw.moe.forward_a2a(comm, xg[r0:r0 + own], T, ws)
            else:
                comm.rs_norm_ag(h, lw.ln2, cfg.rms_eps, T, e)
                act = comm.gemm_ag(lw.gate_up, self.act[:T], T, True, ws)
                e = comm.gemm_rs(act[:, : self.F], lw.down, ws)
            nxt = self.layers[li + 1].ln1 if li + 1 < L else self.norm
            comm.rs_norm_ag(h, nxt, cfg.rms_eps, T, e)
        comm.ag_wait(T)
        B = st.logits_rows.shape[0]
        xs = torch.index_select(xg, 0, m["rows"], out=self.xs[:B])
        return self._lm_head(xs, B)

    def _row_parallel(self, x, w, h):
        self.comm.gemm_allreduce(x, w, h, self.ws)

    def _lm_head(self, xs, B):
        from .. import ops

        if self.lm_head_q is not None:
            loc = ops.w4a16_linear(xs, self.lm_head_q, out=self.logits_local[:B], ws=self.ws)
        else:
            loc = torch.matmul(xs, self.lm_head_dense.T, out=self.logits_local[:B])
        return self.comm.gather_logits(loc, B)


class TorchTPRunner(TorchPagedRunner):
    """CPU fp32 oracle runner over a shard, collectives on gloo. With ``ep_a2a`` MoE layers
    use the expert all-to-all layout of the sequence-parallel GPU mode (csrc/ep_a2a.cu): rank r
    owns rows [r R, r R + own) of the step, routes them, sends each row to the ranks holding its
    experts as (row slot [src][t], local expert id or -1, weight), the receivers run their
    experts over the received slots and return the weighted sums to the row owners, which add
    them up in source order -- here with all_to_all_single, then an all-gather of the owned
    rows (the CPU runner keeps every row on every rank)."""

    def __init__(self, ck: Checkpoint, num_pages: int, comm: TPComm, max_model_len: int = 2048,
                 ep_a2a: bool = False):
        self.comm = comm
        local = shard_checkpoint(ck, comm.rank, comm.tp)
        super().__init__(local, num_pages, max_model_len)
        self.ref.rp_hook = self._rp
        self.ref.head_hook = self._head
        self.ref.reduce_hook = self._reduce
        if ep_a2a and local.config.is_moe:
            self.ref.moe_hook = self._moe_a2a

    def _moe_a2a(self, p: str, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        ref, comm = self.ref, self.comm
        tp, rank = comm.tp, comm.rank
        cfg = ref.cfg
        T, H = x.shape
        K, El, e0 = cfg.num_experts_per_tok, cfg.num_local_experts, cfg.expert_offset
        R = -(-T // tp)
        r0 = rank * R
        own = max(0, min(R, T - r0))
        # dispatch: row slot t of this source in every destination that holds one of its experts
        send_x = torch.zeros(tp, R, H)
        send_id = torch.full((tp, R, K), -1, dtype=torch.int64)
        send_w = torch.zeros(tp, R, K)
        if own:
            topv, topi = ref.route(p, x[r0:r0 + own])
            for t in range(own):
                for k in range(K):
                    e = int(topi[t, k])
                    d = e // El
                    send_x[d, t] = x[r0 + t]
                    send_id[d, t, k] = e - d * El
                    send_w[d, t, k] = topv[t, k]
        recv_x, recv_id, recv_w = torch.empty_like(send_x), torch.empty_like(send_id), torch.empty_like(send_w)
        g = comm.group
        dist.all_to_all_single(recv_x, send_x, group=g)
        dist.all_to_all_single(recv_id, send_id, group=g)
        dist.all_to_all_single(recv_w, send_w, group=g)
        # local experts over the received slots, weighted sums per slot (k in order)
        ys = torch.zeros(tp, R, H)
        for s_ in range(tp):
            for t in range(R):
                for k in range(K):
                    lid = int(recv_id[s_, t, k])
                    if lid >= 0:
                        ys[s_, t] += recv_w[s_, t, k] * ref.expert(p, e0 + lid, recv_x[s_, t])
        back = torch.empty_like(ys)
        dist.all_to_all_single(back, ys, group=g)  # [source rank][my row slot]
        mine = back.sum(0)  # source order
        full = torch.empty(tp * R, H)
        dist.all_gather_into_tensor(full, mine.contiguous(), group=g)
        return full[:T]

    def _reduce(self, part: torch.Tensor) -> torch.Tensor:
        out = torch.zeros_like(part)
        self.comm.allreduce_add(part, out)
        return out

    def _rp(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        out = torch.zeros(x.shape[0], w.shape[0])
        self.comm.gemm_allreduce(x, w, out, None)
        return out

    def _head(self, xs: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return self.comm.gather_logits(xs @ w.T, xs.shape[0]).clone()
