"""LLMEngine: the public inference API (continuous batching over a paged, quantized KV cache).

    eng = LLMEngine.from_preset("qwen2.5-7b", device="cuda")
    rid = eng.add_request(prompt_token_ids, SamplingParams(max_tokens=64))
    while eng.has_unfinished():
        for out in eng.step(): ...

Each ``step()`` schedules one batch (scheduler.py), builds the flat step inputs, runs the
model runner (one H2D copy of the packed metadata, one D2H copy of the sampled token
ids), then appends tokens, applies stop conditions and publishes full KV blocks for
prefix reuse.
"""
from __future__ import annotations

import hashlib
import itertools
import time
import zlib
from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np
import torch

from ..kv.paged import BlockManager, bytes_per_page
from ..models.config import ModelConfig, QuantConfig, get_preset
from ..models.decoder import StepInputs, prefill_tiles
from ..models.weights import Checkpoint, random_checkpoint
from .request import Request, RequestOutput, Status
from .sampling import SamplingParams
from .scheduler import Schedule, ScheduledEntry, Scheduler
from .speculative import TREE_META_INTS, _Guard, make_proposer, spec_eligible


@dataclass
class EngineConfig:
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 2048
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.85
    num_pages: int | None = None
    enable_prefix_caching: bool = True
    cuda_graphs: bool = True
    chunk_align: int = 0
    hist_window: int = 64
    seed: int = 0
    spec: object | None = None  # speculative.SpecConfig: prompt lookup / draft model / Jacobi
    tp: int = 1                 # tensor-parallel ranks (one process per GPU, torch.distributed initialised)
    tp_mode: str = "nvlink"     # "nvlink": fused GEMM+all-reduce over peer memory; "sp": sequence parallel
                                # (fused GEMM->reduce-scatter, RMSNorm+all-gather); "nccl": NCCL baseline
    peer_timeout_s: float = 10.0  # a rank whose heartbeat or liveness is older than this has failed
    kv_host_bytes: int = 0        # > 0: keep evicted prefix blocks in a host-RAM tier of this size
    kv_disk_dir: str | None = None  # spill (and persist across restarts) evicted prefix blocks here
    kv_disk_bytes: int = 8 << 30
    # keep a bf16 expansion of every quantized layer weight resident for prefill GEMMs
    # (>= DQ_GEMM_MIN_M tokens): ~4x the INT4 weight bytes of HBM for no per-step expansion;
    # decode keeps reading the quantized codes
    prefill_weight_cache: bool = True
    # > 0: keep the last-position logits of this many recently prefilled prompts; a request
    # whose prompt repeats one of them gets its first token with no forward pass
    prompt_logit_cache: int = 64
    # attention window (StreamingLLM-style sinks + recent window, page granular): with
    # kv_window_tokens > 0, a sequence keeps its first ceil(kv_sink_tokens / page_size) pages and
    # the pages that hold any of its last kv_window_tokens positions; older pages go back to the
    # pool and attention no longer sees them. 0 = full attention.
    kv_sink_tokens: int = 0
    kv_window_tokens: int = 0
    # heavy-hitter (H2O-style) eviction: keep at most kv_h2o_budget tokens per sequence; when
    # over, the pages outside the sinks and the recent window with the least accumulated
    # attention mass go back to the pool. The mass is measured on the device every
    # kv_h2o_interval decode steps (those steps run outside CUDA graphs). 0 = off.
    kv_h2o_budget: int = 0
    kv_h2o_interval: int = 4
    # score memory: each refresh multiplies a sequence's page scores by this before adding the
    # new mass (1.0 = H2O's accumulated attention; < 1 weights recent queries, the observation
    # window of GreenKV / SnapKV-style scoring with an effective window of 1 / (1 - decay) refreshes)
    kv_h2o_decay: float = 1.0
    # heavy-hitter budgets arbitrated against the page pool (kv/budget.py): every running
    # sequence asks for kv_h2o_budget tokens; when their sum exceeds the pool, each gets a
    # proportional share (never less than its protected sinks + window + one page)
    kv_budget_adaptive: bool = False
    # > 1: the decoder layers split over this many GPUs of this process (cuda:i .. cuda:i+pp-1,
    # from the engine's device), hidden states passed device to device; steps run eagerly
    pp: int = 1
    # > 0: the quantized weights of the last N decoder layers stay in pinned host memory and
    # stream to the GPU one layer ahead of use (models larger than HBM); steps run eagerly
    offload_layers: int = 0
    pp_devices: tuple | None = None  # explicit stage devices (default: consecutive GPUs)


@dataclass
class EngineStats:
    steps: int = 0
    prompt_tokens: int = 0
    generated_tokens: int = 0
    prefix_hit_tokens: int = 0
    preemptions: int = 0
    ttfts: list = field(default_factory=list)
    h2d_bytes: int = 0
    d2h_bytes: int = 0
    graph_steps: int = 0
    mixed_steps: int = 0
    scheduled_tokens: int = 0
    # host seconds per phase of step(): schedule, build (step inputs), run (launches + the wait
    # for the device, the wait alone in runner.sync_wait_s), post (tokens, stops, blocks)
    host_s: dict = field(default_factory=lambda: {"schedule": 0.0, "build": 0.0, "run": 0.0, "post": 0.0})
    # step wall-time histogram (seconds; cumulative counts per upper bound, Prometheus style)
    step_buckets: tuple = (0.002, 0.005, 0.01, 0.02, 0.05, 0.1, 0.25, 1.0, float("inf"))
    step_counts: list = field(default_factory=lambda: [0] * 9)
    step_time_sum: float = 0.0
    instant_first_tokens: int = 0  # first tokens sampled from the prompt-logit cache
    evicted_pages: int = 0         # pages given back by the attention window


class PromptLogitCache:
    """Last-position logits of recently prefilled prompts, keyed by the prompt's token ids
    (LRU over a preallocated [entries, vocab] buffer on the runner's device).

    A request whose prompt is stored gets its first token sampled from the stored row by the
    runner's own sampler, so TTFT is one sampling call instead of a prefill; the prompt (plus
    that token) is then computed by the next steps exactly as for a preempted request that
    resumes, reusing the cached prefix pages. The reference keeps a float32 last-position logit
    per KV block and uses it only when a prompt matches whole blocks to its last token
    (squish/kv/block_kv_cache.py:65-85); here any prompt length qualifies, since the
    uncached tail is computed after the first token is emitted."""

    def __init__(self, entries: int):
        self.entries = entries
        self.buf: torch.Tensor | None = None
        self.slot: OrderedDict[bytes, int] = OrderedDict()
        self.hits = 0

    @staticmethod
    def key(prompt: list[int]) -> bytes:
        return hashlib.blake2b(np.asarray(prompt, dtype=np.int32).tobytes(), digest_size=16).digest()

    def get(self, key: bytes) -> torch.Tensor | None:
        s = self.slot.get(key)
        if s is None:
            return None
        self.slot.move_to_end(key)
        self.hits += 1
        return self.buf[s]

    def put(self, key: bytes, row: torch.Tensor) -> None:
        if key in self.slot:
            self.slot.move_to_end(key)
            return
        if self.buf is None or self.buf.shape[1] != row.shape[0] or self.buf.dtype != row.dtype:
            self.buf = torch.empty(self.entries, row.shape[0], dtype=row.dtype, device=row.device)
            self.slot.clear()
        s = self.slot.popitem(last=False)[1] if len(self.slot) >= self.entries else len(self.slot)
        self.buf[s].copy_(row, non_blocking=True)
        self.slot[key] = s


def _sampling_row(r: Request) -> tuple:
    """(temperature, top_p, min_p, repetition_penalty, top_k) of a request, built once (the
    sampling parameters of a request do not change)."""
    row = r._samp_row
    if row is None:
        p = r.params
        row = r._samp_row = (p.temperature, p.top_p, p.min_p, p.repetition_penalty, float(p.top_k))
    return row


def _rng_base(r: Request) -> int:
    """Per-request sampler stream offset (a hash of the request id, computed once)."""
    b = r._rng_base
    if b is None:
        b = r._rng_base = (zlib.crc32(r.rid.encode()) & 0xFFFF) * 65536
    return b


def _rng_step(r: Request) -> int:
    """Sampler stream position of a request's next token (seeded per request id)."""
    return (r.rng_step + _rng_base(r)) & 0x7FFFFFFF


class LLMEngine:
    def __init__(self, runner, cfg: ModelConfig, qcfg: QuantConfig, ecfg: EngineConfig, num_pages: int):
        self.runner = runner
        self.cfg, self.qcfg, self.ecfg = cfg, qcfg, ecfg
        self.blocks = BlockManager(num_pages, qcfg.page_size, ecfg.enable_prefix_caching, model_key=cfg.name)
        self.scheduler = Scheduler(self.blocks, ecfg.max_num_seqs, ecfg.max_num_batched_tokens, ecfg.max_model_len,
                                   ecfg.chunk_align)
        if ecfg.enable_prefix_caching and (ecfg.kv_host_bytes > 0 or ecfg.kv_disk_dir):
            from ..kv.tiers import KVTierStore, PageIO, layout_of

            rc = getattr(runner, "cfg", cfg)
            self.blocks.tier = KVTierStore(PageIO(runner), layout_of(rc, qcfg), host_bytes=ecfg.kv_host_bytes,
                                           disk_dir=ecfg.kv_disk_dir, disk_bytes=ecfg.kv_disk_bytes)
        self.requests: dict[str, Request] = {}
        self._ids = itertools.count()
        self.kv_broker = None
        if ecfg.kv_h2o_budget > 0 and ecfg.kv_budget_adaptive:
            from ..kv.budget import KVBudgetBroker

            self.kv_broker = KVBudgetBroker(num_pages * qcfg.page_size)
        self.stats = EngineStats()
        self.max_pages = (ecfg.max_model_len + qcfg.page_size - 1) // qcfg.page_size
        self.graphs = None
        self.hidden_states: dict[str, np.ndarray] = {}  # rid -> final hidden of the last prompt token
        self.proposer = None
        self.guard = None
        self.monitor = None   # utils.fault.PeerMonitor (multi-rank engines)
        self.injector = None  # utils.fault.FaultInjector (SQUISH_FAULT)
        self.spec_stats = {"verifies": 0, "drafted": 0, "accepted": 0, "emitted": 0}
        self.logit_cache = PromptLogitCache(ecfg.prompt_logit_cache) if ecfg.prompt_logit_cache > 0 else None
        self._ready: list[RequestOutput] = []  # outputs produced outside a step (cached first tokens)

    # ------------------------------------------------------------------ construction
    @staticmethod
    def plan_pages(cfg: ModelConfig, qcfg: QuantConfig, ecfg: EngineConfig, device) -> int:
        if ecfg.num_pages:
            return ecfg.num_pages
        dev = torch.device(device)
        if dev.type != "cuda":
            return max(64, ecfg.max_num_seqs * ((ecfg.max_model_len + qcfg.page_size - 1) // qcfg.page_size))
        free, total = torch.cuda.mem_get_info(dev)
        budget = free - (1.0 - ecfg.gpu_memory_utilization) * total
        per = bytes_per_page(cfg, qcfg)
        return max(16, int(budget // per))

    @classmethod
    def from_checkpoint(cls, ck: Checkpoint, device="cuda", ecfg: EngineConfig | None = None, **kw) -> "LLMEngine":
        ecfg = ecfg or EngineConfig(**kw)
        dev = torch.device(device)
        # an EAGLE head ties the target's embedding, final norm and LM head (kept before the
        # CUDA runner frees the host copy of the checkpoint)
        keep = None
        if ecfg.spec is not None and ecfg.spec.method in ("eagle", "redrafter"):
            keep = {k: ck.tensors[k] for k in ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight")
                    if k in ck.tensors}
        if ecfg.tp > 1:
            if ecfg.kv_h2o_budget > 0:
                raise ValueError("heavy-hitter KV eviction runs on one GPU per engine (use --dp for more GPUs)")
            if keep is not None:
                raise ValueError("feature-based drafters run on one GPU per engine (use --dp for more GPUs)")
            return cls._from_checkpoint_tp(ck, dev, ecfg)
        if dev.type == "cuda" and ecfg.pp > 1:
            return cls._from_checkpoint_layer_split(ck, dev, ecfg)
        if dev.type == "cuda":
            from ..models.decoder import CudaRunner

            # weights first, then size the page pool from what is left
            spec_rows = ecfg.max_num_seqs * ecfg.spec.max_nodes if ecfg.spec is not None else 0
            runner = CudaRunner(ck, dev, num_pages=1, max_num_tokens=ecfg.max_num_batched_tokens,
                                max_num_seqs=ecfg.max_num_seqs, max_model_len=ecfg.max_model_len,
                                free_checkpoint=True, spec_rows=spec_rows,
                                prefill_weight_cache=ecfg.prefill_weight_cache and not ecfg.offload_layers,
                                offload_layers=ecfg.offload_layers)
            if ecfg.offload_layers:
                import dataclasses

                ecfg = dataclasses.replace(ecfg, cuda_graphs=False)  # (side-stream copies each step)
            del runner.pools
            torch.cuda.empty_cache()
            num_pages = cls.plan_pages(ck.config, ck.quant, ecfg, dev)
            from ..kv.paged import KVPools

            runner.pools = KVPools(ck.config, ck.quant, num_pages, dev)
        else:
            from ..models.decoder import TorchPagedRunner

            num_pages = cls.plan_pages(ck.config, ck.quant, ecfg, dev)
            runner = TorchPagedRunner(ck, num_pages, ecfg.max_model_len)
        eng = cls(runner, ck.config, ck.quant, ecfg, num_pages)
        eng.checkpoint_tensors = keep
        if dev.type == "cuda" and ecfg.cuda_graphs:
            from .cuda_graph import DecodeGraphs

            eng.graphs = DecodeGraphs(eng)
        if ecfg.spec is not None:
            eng.proposer = make_proposer(ecfg.spec, eng)
            eng.guard = _Guard(ecfg.spec.miss_limit, ecfg.spec.cooldown) if ecfg.spec.adaptive else None
        return eng

    @classmethod
    def _from_checkpoint_layer_split(cls, ck: Checkpoint, dev: torch.device, ecfg: EngineConfig) -> "LLMEngine":
        """Layer-split engine: the layers over ecfg.pp GPUs of this process (the pool of every
        stage has the same page count; each stage holds only its layers' pages)."""
        import dataclasses

        from ..kv.paged import KVPools
        from ..models.decoder import LayerSplitRunner

        if ecfg.spec is not None or ecfg.kv_h2o_budget > 0 or ecfg.kv_host_bytes > 0 or ecfg.kv_disk_dir:
            raise ValueError("the layer split serves plain decoding (no speculation, H2O eviction or KV tiers)")
        base = dev.index or 0
        devs = ([torch.device(d) for d in ecfg.pp_devices] if ecfg.pp_devices else
                [torch.device("cuda", base + i) for i in range(ecfg.pp)])
        runner = LayerSplitRunner(ck, devs, 1, max_num_tokens=ecfg.max_num_batched_tokens,
                                  max_num_seqs=ecfg.max_num_seqs, max_model_len=ecfg.max_model_len,
                                  prefill_weight_cache=ecfg.prefill_weight_cache)
        for st_ in runner.stages:
            del st_.pools
        torch.cuda.empty_cache()
        if ecfg.num_pages:
            num_pages = ecfg.num_pages
        else:  # the tightest stage decides (its layers' bytes per page against its free memory)
            num_pages = None
            for st_, d in zip(runner.stages, devs):
                free, total = torch.cuda.mem_get_info(d)
                per = bytes_per_page(st_.cfg, ck.quant)
                n = int((free - (1.0 - ecfg.gpu_memory_utilization) * total) // per)
                num_pages = n if num_pages is None else min(num_pages, n)
            num_pages = max(16, num_pages)
        for st_, d in zip(runner.stages, devs):
            st_.pools = KVPools(st_.cfg, ck.quant, num_pages, d)
        return cls(runner, ck.config, ck.quant, dataclasses.replace(ecfg, cuda_graphs=False), num_pages)

    @classmethod
    def _from_checkpoint_tp(cls, ck: Checkpoint, dev: torch.device, ecfg: EngineConfig) -> "LLMEngine":
        """Tensor-parallel engine: this process holds one shard; every rank runs the same
        host logic (scheduling is deterministic and every rank samples the same tokens)."""
        import torch.distributed as dist

        from ..kv.paged import KVPools
        from ..parallel.comm import TPComm

        if not dist.is_initialized() or dist.get_world_size() != ecfg.tp:
            raise RuntimeError(f"tp={ecfg.tp} needs torch.distributed initialised with {ecfg.tp} ranks")
        cfg = ck.config
        spec_rows = ecfg.max_num_seqs * ecfg.spec.max_nodes if ecfg.spec is not None else 0
        rows = ecfg.max_num_seqs + min(ecfg.max_num_batched_tokens, spec_rows)
        if dev.type == "cuda":
            from ..parallel.tp_runner import TPCudaRunner

            comm = TPComm(ecfg.tp_mode, ecfg.max_num_batched_tokens, cfg.hidden_size, rows, cfg.vocab_size,
                          device=dev)
            runner = TPCudaRunner(ck, dev, 1, comm, max_num_tokens=ecfg.max_num_batched_tokens,
                                  max_num_seqs=ecfg.max_num_seqs, max_model_len=ecfg.max_model_len,
                                  free_checkpoint=True, spec_rows=spec_rows,
                                  prefill_weight_cache=ecfg.prefill_weight_cache)
            del runner.pools
            torch.cuda.empty_cache()
            pages = torch.tensor([cls.plan_pages(runner.cfg, ck.quant, ecfg, dev)], device=dev)
            dist.all_reduce(pages, op=dist.ReduceOp.MIN)  # identical pools -> identical scheduling
            num_pages = int(pages.item())
            runner.pools = KVPools(runner.cfg, ck.quant, num_pages, dev)
        else:
            from ..parallel.tp_runner import TorchTPRunner

            comm = TPComm("cpu", ecfg.max_num_batched_tokens, cfg.hidden_size, rows, cfg.vocab_size)
            num_pages = cls.plan_pages(cfg, ck.quant, ecfg, dev)
            runner = TorchTPRunner(ck, num_pages, comm, ecfg.max_model_len, ep_a2a=ecfg.tp_mode == "sp")
        eng = cls(runner, cfg, ck.quant, ecfg, num_pages)
        eng.comm = comm
        from ..utils.fault import FaultInjector, PeerMonitor

        rank = dist.get_rank()
        eng.injector = FaultInjector(rank)
        eng.monitor = PeerMonitor(dist.distributed_c10d._get_default_store(), rank, dist.get_world_size(),
                                  timeout_s=ecfg.peer_timeout_s, injector=eng.injector).start_liveness()
        if dev.type == "cuda" and ecfg.cuda_graphs:
            from .cuda_graph import DecodeGraphs

            eng.graphs = DecodeGraphs(eng)
        if ecfg.spec is not None:
            eng.proposer = make_proposer(ecfg.spec, eng)
            eng.guard = _Guard(ecfg.spec.miss_limit, ecfg.spec.cooldown) if ecfg.spec.adaptive else None
        return eng

    @classmethod
    def from_preset(cls, name: str, device="cuda", seed: int = 0, ecfg: EngineConfig | None = None,
                    **kw) -> "LLMEngine":
        cfg, q = get_preset(name)
        dev = torch.device(device)
        ck = random_checkpoint(cfg, q, seed=seed, device=dev)
        return cls.from_checkpoint(ck, dev, ecfg, **kw)

    def close(self) -> None:
        """Persist the host KV tier to disk (when a disk tier is configured)."""
        if self.blocks.tier is not None:
            self.blocks.tier.flush()

    def save_session(self, tokens: list[int]) -> int:
        """Copy the cached KV blocks of a conversation (its prompt + output tokens, full blocks
        only) into the host / disk tiers now, rather than when their pages are reused, and write
        the host tier to disk: a later request with the same prefix (this process or a restarted
        one on the same disk directory) restores them instead of recomputing. Returns the blocks
        saved. The reference keeps per-session KV files (squish/kv/kv_cache.py:3263-3560,
        ``SessionKVCache`` / ``DiskKVCache``); here sessions are the chained-hash blocks."""
        from ..kv.paged import chain_hashes

        tier = self.blocks.tier
        if tier is None:
            raise ValueError("saving a session needs a KV tier (kv_host_bytes or kv_disk_dir)")
        n = 0
        for h in chain_hashes(tokens, self.qcfg.page_size, self.blocks.model_key):
            p = self.blocks.hash_to_page.get(h)
            if p is None:
                if tier.has(h):
                    continue
                break  # the chain is broken here: later blocks cannot be matched anyway
            if not tier.has(h):
                tier.offload(h, p)
                n += 1
        tier.flush()
        return n

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt: list[int], params: SamplingParams | None = None, rid: str | None = None) -> str:
        params = (params or SamplingParams()).validate()
        if not prompt:
            raise ValueError("empty prompt")
        lo, hi = min(prompt), max(prompt)
        if lo < 0 or hi >= self.cfg.vocab_size:
            raise ValueError(f"token id out of range [0, {self.cfg.vocab_size}): {lo if lo < 0 else hi}")
        rid = rid or f"req-{next(self._ids)}"
        req = Request(rid, list(map(int, prompt)), params)
        self.scheduler.add(req)
        self.requests[rid] = req
        if self.logit_cache is not None:
            req.prompt_key = self.logit_cache.key(req.prompt)
            if params.grammar is None and not params.return_hidden and not params.logprobs:
                self._instant_first_token(req)
        return rid

    def _instant_first_token(self, req: Request) -> None:
        """Sample the first token from the prompt-logit cache (no forward pass) on a hit."""
        row = self.logit_cache.get(req.prompt_key)
        if row is None:
            return
        p = req.params
        hist = None
        if p.repetition_penalty != 1.0:
            hist = np.full((1, self.ecfg.hist_window), -1, dtype=np.int32)
            t = req.prompt[-self.ecfg.hist_window:]
            hist[0, :len(t)] = t
        tok = self.runner.sample_row(row, p.temperature, p.top_p, p.top_k, p.min_p, p.repetition_penalty, hist,
                                     self.ecfg.seed, _rng_step(req))
        self.stats.instant_first_tokens += 1
        out = self._emit(req, [tok], time.perf_counter())
        if out.finished and req in self.scheduler.waiting:
            self.scheduler.waiting.remove(req)
        self._ready.append(out)

    def abort(self, rid: str) -> None:
        req = self.requests.get(rid)
        if req is None or req.status is Status.FINISHED:
            return
        if req in self.scheduler.waiting:
            self.scheduler.waiting.remove(req)
            req.status = Status.FINISHED
            req.finish_reason = "abort"
        else:
            self.scheduler.finish(req, "abort")

    def warmup_graphs(self, batch: int | None = None) -> int:
        """Capture the decode CUDA graphs a steady state of ``batch`` sequences (default
        max_num_seqs) replays, for every context bucket up to max_model_len, then freeze the
        objects alive so far out of the cyclic garbage collector's scans. Call after loading,
        before serving; returns the number of graphs captured."""
        import gc

        n = 0
        if self.graphs is not None:
            n = self.graphs.prewarm(batch or self.ecfg.max_num_seqs, self.ecfg.max_model_len)
        gc.collect()
        gc.freeze()
        return n

    def has_unfinished(self) -> bool:
        return bool(self._ready) or self.scheduler.has_work()

    # ------------------------------------------------------------------ step
    def build_inputs(self, sched: Schedule) -> StepInputs:
        ps = self.qcfg.page_size
        entries = sched.decode + sched.prefill
        T = sum(e.n for e in entries)
        ids = np.empty(T, dtype=np.int32)
        pos = np.empty(T, dtype=np.int32)
        slots = np.empty(T, dtype=np.int32)
        nb = len(entries)
        if self.graphs is not None:
            maxp = self.max_pages
        else:
            maxp = max((len(e.req.page_array()) for e in entries), default=1)
        bt = np.zeros((nb, max(maxp, 1)), dtype=np.int32)
        rows, samp = [], []
        trees = [e for e in entries if e.tree is not None]
        tmask = np.zeros(T, dtype=np.int32) if trees else None
        vrows, vmeta, vreqs = [], [], []
        off = 0
        for i, e in enumerate(entries):
            r = e.req
            pg = r.page_array()
            bt[i, :len(pg)] = pg
            if r.evicted_tokens:
                pg = r.logical_pages()
            if e.n == 1 and e.tree is None:  # decode: scalars, no per-entry numpy temporaries
                ids[off] = r.token_at(e.start)
                pos[off] = e.start
                slots[off] = r.pages[e.start // ps] * ps + e.start % ps
                if e.sample:
                    rows.append(off)
                    samp.append(r)
                off += 1
                continue
            if e.tree is not None:
                tr = e.tree
                ids[off:off + e.n] = tr.tokens
                pos[off:off + e.n] = e.start + np.asarray(tr.depth, dtype=np.int32)
                p = np.arange(e.start, e.start + e.n, dtype=np.int32)
                slots[off:off + e.n] = pg[p // ps] * ps + p % ps
                tmask[off:off + e.n] = tr.masks()
                vmeta.append(tr.meta_row(len(vrows)))
                vrows.extend(range(off, off + e.n))
                vreqs.append(r)
                off += e.n
                continue
            ids[off:off + e.n] = r.token_slice(e.start, e.n)
            p = np.arange(e.start, e.start + e.n, dtype=np.int32)
            pos[off:off + e.n] = p
            slots[off:off + e.n] = pg[p // ps] * ps + p % ps
            if e.sample:
                rows.append(off + e.n - 1)
                samp.append(r)
            off += e.n
        nd = len(sched.decode)
        dl = np.asarray([e.start + 1 - e.req.evicted_tokens for e in sched.decode], dtype=np.int32)
        ql = np.asarray([e.n for e in sched.prefill], dtype=np.int32)
        ctx = np.asarray([e.start + e.n - e.req.evicted_tokens for e in sched.prefill], dtype=np.int32)
        qs = np.zeros(len(ql), dtype=np.int32)
        if len(ql):
            qs[1:] = np.cumsum(ql)[:-1]
        tseq, tq0 = prefill_tiles(ql)
        B = len(samp)
        # one pass over the sampled requests: (temperature, top_p, min_p, penalty) and top_k
        pf = np.array([_sampling_row(r) for r in samp], dtype=np.float32).reshape(B, 5)
        temp, topp, minp, rep = pf[:, 0].copy(), pf[:, 1].copy(), pf[:, 2].copy(), pf[:, 3].copy()
        topk = pf[:, 4].astype(np.int32)

        def rng_steps(reqs):
            return np.asarray([_rng_step(r) for r in reqs], dtype=np.int64).astype(np.int32)

        step = rng_steps(samp)
        hist = None
        if B and (rep != 1.0).any():
            hw = self.ecfg.hist_window
            hist = np.full((B, hw), -1, dtype=np.int32)
            for i, r in enumerate(samp):
                t = r.tokens[-hw:]
                hist[i, :len(t)] = t
        mask = None
        if B and any(r.params.grammar is not None for r in samp):
            words = (self.cfg.vocab_size + 31) // 32
            mask = np.full((B, words), -1, dtype=np.int32)
            for i, r in enumerate(samp):
                if r.params.grammar is not None:
                    mask[i] = np.asarray(r.params.grammar.allowed_mask(), dtype=np.uint32).view(np.int32)[:words]
        st = StepInputs(ids, pos, slots, nd, dl, qs, ql, ctx, tseq, tq0, bt,
                        np.asarray(rows + vrows, dtype=np.int32), temp, topp, topk, minp, rep, step, hist,
                        self.ecfg.seed, int(dl.max()) if nd else 0)
        st.allow_mask = mask
        if trees:
            st.tree_mask = tmask
            st.verify_meta = np.stack(vmeta).astype(np.int32)
            st.verify_temp = np.asarray([r.params.temperature for r in vreqs], dtype=np.float32)
            st.verify_step = rng_steps(vreqs)
            st.verify_preds = bool(getattr(self.proposer, "wants_preds", False))
            st.draft_logits = getattr(self.proposer, "qbuf", None)
        return st, samp

    def run_entries(self, decode: list[ScheduledEntry], prefill: list[ScheduledEntry]) -> np.ndarray:
        """Run one forward over explicit entries (used by a draft model's proposer); returns the
        sampled token of every sampling entry; logits stay in ``runner.logits``."""
        st, _ = self.build_inputs(Schedule(decode, prefill, []))
        if self.graphs is not None and not prefill and self.graphs.can_run(st):
            return self.graphs.run(st)
        return self.runner.execute(st)

    def _attach_drafts(self, sched: Schedule) -> None:
        """Turn decode entries with a draft tree into verification chunks (prefill group)."""
        sc = self.ecfg.spec
        cands = [e.req for e in sched.decode if spec_eligible(e.req.params) and
                 (self.guard is None or self.guard.allow(e.req.rid))]
        if not cands:
            return
        trees = self.proposer.propose(cands)
        if not trees:
            return
        budget = min(self.ecfg.max_num_batched_tokens, getattr(self.runner, "max_num_tokens", 1 << 30))
        used = sum(e.n for e in sched.decode + sched.prefill)
        cap_rows = getattr(self.runner, "spec_rows", 1 << 30)
        rows = 0
        verify = []
        for e in list(sched.decode):
            t = trees.get(e.req.rid)
            if t is None or t.size < 2:
                continue
            n = min(t.size, sc.max_nodes)
            if used + n - 1 > budget or rows + n > cap_rows:
                break
            if not self.scheduler._ensure_pages(e.req, e.start + n):
                continue
            if n < t.size:  # parents precede children, so a prefix of the nodes is a tree
                t = type(t)(t.tokens[:n], t.parent[:n], t.qrow[:n])
            e.n, e.tree = n, t
            sched.decode.remove(e)
            verify.append(e)
            used += n - 1
            rows += n
        sched.prefill[:0] = verify

    def step(self) -> list[RequestOutput]:
        if self._ready:  # first tokens sampled at submission: returned before any forward runs
            ready, self._ready = self._ready, []
            return ready
        return self._step_guarded()

    def _step_guarded(self) -> list[RequestOutput]:
        if self.monitor is None and self.injector is None:
            return self._step()
        n = self.stats.steps
        try:
            if self.injector is not None:
                self.injector.before_step(n, on_hang=self.monitor.stop_liveness if self.monitor else None)
            if self.monitor is not None:
                self.monitor.check()  # fail fast, before this step's collectives
            outs = self._step()
        except Exception as exc:
            if self.monitor is not None:
                self.monitor.announce_error(f"{type(exc).__name__}: {exc}")
            raise
        if self.monitor is not None:
            self.monitor.beat(n + 1)
        return outs

    def _step(self) -> list[RequestOutput]:
        hs = self.stats.host_s
        t0 = time.perf_counter()
        sched = self.scheduler.schedule()
        self.stats.preemptions += len(sched.preempted)
        if sched.empty:
            return []
        if self.proposer is not None and sched.decode:
            self._attach_drafts(sched)
        t1 = time.perf_counter()
        st, samp = self.build_inputs(sched)
        t2 = time.perf_counter()
        score = self._h2o_score_step(sched)
        self.runner.score_step = score
        if (self.graphs is not None and not sched.prefill and st.allow_mask is None and st.num_verify == 0
                and not score and self.graphs.can_run(st)):
            toks = self.graphs.run(st)
            self.stats.graph_steps += 1
        else:
            toks = self.runner.execute(st)
            self.stats.mixed_steps += 1 if sched.prefill else 0
        self.runner.score_step = False
        t3 = time.perf_counter()
        hs["schedule"] += t1 - t0
        hs["build"] += t2 - t1
        hs["run"] += t3 - t2
        self.stats.scheduled_tokens += st.num_tokens
        self.stats.steps += 1
        self.stats.h2d_bytes += st.h2d_bytes()
        self.stats.d2h_bytes += 4 * len(samp) + 4 * st.num_verify * (2 + 32)
        now = time.perf_counter()
        outs: list[RequestOutput] = []
        # advance computed counters, publish full blocks
        for e in sched.decode + sched.prefill:
            r = e.req
            if e.tree is None:
                r.num_computed = e.start + e.n
                if not e.sample:
                    self.stats.prompt_tokens += e.n
        if self.logit_cache is not None:  # first tokens: keep the prompt's last-position logits
            for i, r in enumerate(samp):
                if not r.output and r.prompt_key is not None:
                    self.logit_cache.put(r.prompt_key, self.runner.logit_row(i))
        want_hidden = [i for i, r in enumerate(samp) if r.params.return_hidden]
        if want_hidden:
            hid = self.runner.last_hidden
            for i in want_hidden:
                self.hidden_states[samp[i].rid] = hid[i].float().cpu().numpy()
        for r, t in zip(samp, toks.tolist()):
            outs.append(self._emit(r, [int(t)], now))
        self._hid_rows = [(r, i) for i, r in enumerate(samp)]
        if st.num_verify:
            outs.extend(self._apply_verify(sched, st, now))
        if getattr(self.proposer, "wants_hidden", False):
            self._observe_hidden()
        if score:
            self._h2o_collect(sched)
        t4 = time.perf_counter()
        hs["post"] += t4 - t3
        dt = t4 - t0
        self.stats.step_time_sum += dt
        for i, b in enumerate(self.stats.step_buckets):
            if dt <= b:
                self.stats.step_counts[i] += 1
        if self.ecfg.kv_h2o_budget > 0:
            if self.kv_broker is not None:
                self._sync_budgets()
            for e in sched.decode:
                if e.req.status is Status.RUNNING:
                    self._evict_h2o(e.req)
        elif self.ecfg.kv_window_tokens > 0:
            for e in sched.decode + sched.prefill:
                if e.req.status is Status.RUNNING:
                    self._evict_window(e.req)
        return outs

    # ------------------------------------------------------------------ heavy-hitter eviction
    def _h2o_score_step(self, sched: Schedule) -> bool:
        if self.ecfg.kv_h2o_budget <= 0 or not sched.decode or self.stats.steps % max(1, self.ecfg.kv_h2o_interval):
            return False
        # refresh while some decoding sequence is near its budget
        return any(e.req.num_computed - e.req.evicted_tokens > self.h2o_budget(e.req) // 2 for e in sched.decode)

    def _h2o_collect(self, sched: Schedule) -> None:
        """Add this step's attention mass per page (all layers and heads) to each decoding
        sequence's per-page totals."""
        mass = self.runner.page_mass_buf
        reqs = [e.req for e in sched.decode if e.tree is None]
        if not reqs:
            return
        idx = [np.flatnonzero(np.asarray(r.pages) >= 0) for r in reqs]
        phys = np.concatenate([np.asarray(r.pages, dtype=np.int64)[i] for r, i in zip(reqs, idx)])
        vals = mass[torch.from_numpy(phys).to(mass.device)].float().cpu().numpy()
        off = 0
        for r, i in zip(reqs, idx):
            if r.h2o_mass is None or len(r.h2o_mass) < len(r.pages):
                grown = np.zeros(max(len(r.pages), 16) * 2, dtype=np.float64)
                if r.h2o_mass is not None:
                    grown[:len(r.h2o_mass)] = r.h2o_mass
                r.h2o_mass = grown
            if self.ecfg.kv_h2o_decay != 1.0:
                r.h2o_mass *= self.ecfg.kv_h2o_decay
            r.h2o_mass[i] += vals[off:off + len(i)]
            off += len(i)
            r.h2o_scored = len(r.pages)

    def _sync_budgets(self) -> None:
        """One broker registration per running sequence (kv_h2o_budget tokens each)."""
        br = self.kv_broker
        live = {f"h2o:{r.rid}" for r in self.scheduler.running}
        for name in [n for n in br.names() if n not in live]:
            br.unregister(name)
        for name in sorted(live - set(br.names())):
            br.register(name, self.ecfg.kv_h2o_budget)

    def h2o_budget(self, r: Request) -> int:
        """Tokens sequence ``r`` may keep: kv_h2o_budget, or its arbitrated share."""
        ec = self.ecfg
        name = f"h2o:{r.rid}"
        if self.kv_broker is None or name not in self.kv_broker.names():
            return ec.kv_h2o_budget
        floor = ec.kv_sink_tokens + max(ec.kv_window_tokens, self.qcfg.page_size) + self.qcfg.page_size
        return max(floor, self.kv_broker.allocated(name))

    def _evict_h2o(self, r: Request) -> None:
        """Over budget: give back the scored pages outside the sinks and the recent window with
        the least accumulated attention mass (only full pages scored at least once)."""
        ps, ec = self.qcfg.page_size, self.ecfg
        over = r.num_computed - r.evicted_tokens - self.h2o_budget(r)
        if over <= 0 or r.h2o_mass is None:
            return
        sink = -(-ec.kv_sink_tokens // ps)
        recent = (r.num_computed - max(ec.kv_window_tokens, ps)) // ps  # pages [recent, ..) are protected
        cand = [b for b in range(sink, min(recent, r.h2o_scored)) if r.pages[b] >= 0]
        if not cand:
            return
        cand.sort(key=lambda b: (r.h2o_mass[b], b))
        gone = cand[:-(-over // ps)]
        self.blocks.release([r.pages[b] for b in gone])
        for b in gone:
            r.pages[b] = -1
            r.evicted_at[b] = r.num_computed
        r.evicted_tokens += len(gone) * ps
        self.stats.evicted_pages += len(gone)

    def _evict_window(self, r: Request) -> None:
        """Give back the pages between the sink pages and the recent window (page granular:
        a page goes when its last position is older than the window)."""
        ps = self.qcfg.page_size
        sink = -(-self.ecfg.kv_sink_tokens // ps)
        upto = (r.num_computed - self.ecfg.kv_window_tokens) // ps  # pages [.., upto) are out of the window
        start = max(sink, r.evict_from)
        if upto <= start:
            return
        gone = [p for p in r.pages[start:upto] if p >= 0]
        for b in range(start, upto):
            r.pages[b] = -1
        self.blocks.release(gone)
        r.evicted_tokens += len(gone) * ps
        r.evict_from = upto
        self.stats.evicted_pages += len(gone)

    def _emit(self, r: Request, new: list[int], now: float) -> RequestOutput:
        """Append tokens to a request (stopping early at a stop condition)."""
        got = []
        reason = None
        for t in new:
            if r.params.grammar is not None:
                r.params.grammar.advance(int(t))
            if r.first_token_time is None:
                r.first_token_time = now
                self.stats.ttfts.append(now - r.arrival)
                self.stats.prefix_hit_tokens += r.prefix_hit_tokens
            r.output.append(int(t))
            r.rng_step += 1
            self.stats.generated_tokens += 1
            got.append(int(t))
            reason = self._stop_reason(r, int(t))
            if reason:
                break
        self._publish_blocks(r)
        if reason:
            self.scheduler.finish(r, reason)
            r.finish_time = now
            if self.proposer is not None:
                self.proposer.forget(r.rid)
                if self.guard is not None:
                    self.guard.forget(r.rid)
        return RequestOutput(r.rid, got, reason is not None, reason, len(r.prompt), len(r.output))

    def _apply_verify(self, sched: Schedule, st: StepInputs, now: float) -> list[RequestOutput]:
        res = self.runner.last_verify
        preds = getattr(self.runner, "last_preds", None)
        ps = self.qcfg.page_size
        src, dst, outs = [], [], []
        vrow = 0
        g = 0
        fa = self.ecfg.spec.force_accept
        for e in sched.prefill:
            if e.tree is None:
                continue
            r, tr = e.req, e.tree
            nacc, final = int(res[g, 0]), int(res[g, 1])
            path = [int(x) for x in res[g, 2:2 + nacc]]
            if fa is not None:  # benchmark knob: pretend the first chain matched exactly fa drafts
                chain, u = [], 0
                while len(chain) < fa:
                    kids = [c for c in range(1, tr.size) if tr.parent[c] == u]
                    if not kids:
                        break
                    u = kids[0]
                    chain.append(u)
                path, nacc = chain, len(chain)
            toks = [tr.tokens[c] for c in path] + [final]
            for j, c in enumerate(path):
                if c != j + 1:
                    a, b = e.start + c, e.start + j + 1
                    src.append(r.pages[a // ps] * ps + a % ps)
                    dst.append(r.pages[b // ps] * ps + b % ps)
            r.num_computed = e.start + nacc + 1
            self.spec_stats["verifies"] += 1
            self.spec_stats["drafted"] += tr.size - 1
            self.spec_stats["accepted"] += nacc
            self.spec_stats["emitted"] += nacc + 1
            if self.guard is not None:
                self.guard.record(r.rid, nacc)
            p_ = None if preds is None else preds[vrow:vrow + tr.size]
            self.proposer.after_verify(r, nacc, p_)
            # the final token came from the last accepted node's row (after the sampled rows)
            self._hid_rows.append((r, st.num_sample_rows + vrow + (path[-1] if path else 0)))
            vrow += tr.size
            g += 1
            outs.append(self._emit(r, toks, now))
        if src:
            self.runner.kv_compact(src, dst)
        return outs

    def _observe_hidden(self) -> None:
        """Hand the hidden-state proposer (Medusa heads) the final-norm rows that produced each
        live request's newest token."""
        live = [(r, i) for r, i in self._hid_rows if r.finish_time is None]
        if not live:
            return
        hid = self.runner.last_hidden
        rows = [i for _, i in live]
        if max(rows) >= hid.shape[0]:  # checked on the host: a bad row must not reach a device gather
            raise RuntimeError(f"hidden row {max(rows)} outside the step's {hid.shape[0]} logits rows")
        idx = torch.tensor(rows, dtype=torch.long, device=hid.device)
        self.proposer.observe([r for r, _ in live], hid.index_select(0, idx))

    def _publish_blocks(self, r: Request) -> None:
        full = r.num_computed // self.qcfg.page_size
        if full > r.registered_blocks:
            r.chain_hash = self.blocks.register_blocks(r.tokens, r.pages, r.registered_blocks,
                                                       full - r.registered_blocks, r.chain_hash)
            r.registered_blocks = full

    def _stop_reason(self, r: Request, tok: int) -> str | None:
        p = r.params
        n = len(r.output)
        if n >= p.min_tokens:
            if not p.ignore_eos and tok == self.cfg.eos_token_id:
                return "stop"
            if tok in p.stop_token_ids:
                return "stop"
            if p.grammar is not None and getattr(p.grammar, "is_terminated", lambda: False)():
                return "stop"
        if n >= p.max_tokens:
            return "length"
        if r.total_len >= self.ecfg.max_model_len:
            return "length"
        return None

    # ------------------------------------------------------------------ convenience
    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams] | None = None
                 ) -> list[list[int]]:
        ps = params if isinstance(params, list) else [params] * len(prompts)
        rids = [self.add_request(p, sp) for p, sp in zip(prompts, ps)]
        while self.has_unfinished():
            self.step()
        return [self.requests[r].output for r in rids]
