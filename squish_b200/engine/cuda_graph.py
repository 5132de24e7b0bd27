"""CUDA graphs for decode-only steps.

A decode step launches ~10 kernels per layer; replaying a captured graph removes the
per-launch host cost. Graphs are captured lazily per (batch bucket, context bucket):
the batch is padded to the bucket with inert rows (slot -1: no KV write; one visible
token; greedy; logits discarded) and the flash-decoding split count is fixed by the
context bucket. All buffers the graph touches are static: the runner's activation
buffers, the packed metadata staging area (identical offsets for a given bucket, since
every array's size is a function of the bucket alone) and the per-device workspace.
The reference compiles its MLX decode step with mx.compile (squish/server.py:2385-2399);
this is the CUDA counterpart.
"""
from __future__ import annotations

import gc

import numpy as np
import torch

from ..models.decoder import StepInputs
from ..ops.kernels import LAUNCHES

BATCH_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 128, 160, 192, 256)


def _ctx_bucket(n: int) -> int:
    b = 256
    while b < n:
        b *= 2
    return b


class DecodeGraphs:
    def __init__(self, engine):
        self.eng = engine
        self.runner = engine.runner
        self.max_batch = min(engine.ecfg.max_num_seqs, self.runner.max_num_seqs)
        self.graphs: dict[tuple[int, int], tuple[torch.cuda.CUDAGraph, dict]] = {}
        self.pool = None
        self.enabled = True

    def can_run(self, st: StepInputs) -> bool:
        return (self.enabled and st.num_prefill == 0 and st.num_decode == st.num_tokens and
                0 < st.num_decode <= self.max_batch and not st.all_logits)

    def _pad(self, st: StepInputs, bucket: int, ctxb: int) -> StepInputs:
        B = st.num_decode
        pad = bucket - B
        hw = self.eng.ecfg.hist_window

        def p(a, fill, dt):
            return np.concatenate([a.astype(dt), np.full(pad, fill, dtype=dt)]) if pad else a.astype(dt)

        bt = np.zeros((bucket, self.eng.max_pages), dtype=np.int32)
        bt[:B, :st.block_tables.shape[1]] = st.block_tables
        hist = np.full((bucket, hw), -1, dtype=np.int32)
        if st.hist is not None:
            hist[:B] = st.hist
        e = np.zeros(0, dtype=np.int32)
        return StepInputs(
            p(st.input_ids, 0, np.int32), p(st.positions, 0, np.int32), p(st.slot_mapping, -1, np.int32), bucket,
            p(st.decode_seq_lens, 1, np.int32), e, e, e, e, e, bt, np.arange(bucket, dtype=np.int32),
            p(st.temperature, 0.0, np.float32), p(st.top_p, 1.0, np.float32), p(st.top_k, 0, np.int32),
            p(st.min_p, 0.0, np.float32), p(st.rep_penalty, 1.0, np.float32), p(st.rng_step, 0, np.int32), hist,
            st.seed, ctxb)

    def _capture(self, st: StepInputs):
        r = self.runner
        m = r.upload(st)
        s = torch.cuda.Stream(device=r.device)
        s.wait_stream(torch.cuda.current_stream(r.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm up (sets kernel attributes, fills caches)
                logits = r.forward(st, m)
                r.sample_full(st, m, logits)
        torch.cuda.current_stream(r.device).wait_stream(s)
        torch.cuda.synchronize(r.device)
        g = torch.cuda.CUDAGraph()
        r.ws.frozen = True
        before = LAUNCHES[0]
        # A cyclic garbage collection during capture could destroy an unreachable engine's
        # graphs (cudaGraphExecDestroy), which is not permitted while a stream captures and
        # invalidates this capture: collect first, keep the collector off until capture ends.
        gc.collect()
        gc.disable()
        try:
            with torch.cuda.graph(g, pool=self.pool):
                logits = r.forward(st, m)
                toks = r.sample_full(st, m, logits)
        finally:
            gc.enable()
        n_kernels = LAUNCHES[0] - before
        if self.pool is None:
            self.pool = g.pool()
        return g, {"tokens": toks, "launches": n_kernels}

    @torch.inference_mode()
    def prewarm(self, batch: int, max_len: int) -> int:
        """Capture the graphs of ``batch`` decoding sequences for every context bucket up to
        ``max_len`` ahead of time (inert rows), so no capture, with its garbage collection, runs
        inside a serving step. Returns the number of graphs captured."""
        bucket = next((b for b in BATCH_BUCKETS if b >= min(batch, self.max_batch)), None)
        if bucket is None or not self.enabled:
            return 0
        e, f = np.zeros(0, dtype=np.int32), np.zeros(0, dtype=np.float32)
        st0 = StepInputs(e, e, e, 0, e, e, e, e, e, e, np.zeros((0, 1), dtype=np.int32), e, f, f, e, f, f, e, None,
                         self.eng.ecfg.seed, 1)
        n = 0
        ctxb = 256
        while True:
            if (bucket, ctxb) not in self.graphs:
                self.graphs[(bucket, ctxb)] = self._capture(self._pad(st0, bucket, ctxb))
                n += 1
            if ctxb >= max_len:
                break
            ctxb *= 2
        return n

    @torch.inference_mode()
    def run(self, st: StepInputs) -> np.ndarray:
        B = st.num_decode
        bucket = next(b for b in BATCH_BUCKETS if b >= B)
        ctxb = _ctx_bucket(max(st.max_decode_ctx, 1))
        ps = self._pad(st, bucket, ctxb)
        key = (bucket, ctxb)
        r = self.runner
        if key not in self.graphs:
            self.graphs[key] = self._capture(ps)
        g, out = self.graphs[key]
        r.timer_start()
        r.upload(ps)  # same sizes -> same offsets as at capture time
        g.replay()
        LAUNCHES[0] += out["launches"]
        toks = out["tokens"]
        r.tokens_host[:bucket].copy_(toks, non_blocking=True)
        r.timer_stop()
        r.sync()
        r.last_hidden = r.xs[:B]  # final-norm rows of the replayed step (static buffer)
        return r.tokens_host[:B].numpy().copy()
