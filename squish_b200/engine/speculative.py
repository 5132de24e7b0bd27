"""Speculative decoding: draft token trees, proposers, and the verification bookkeeping.

Each decoding request with a draft is verified in the same engine step as everything else:
its tree (node 0 = the pending token, up to 32 nodes, parents before children) is scheduled
as one prefill-style chunk with a token-tree attention mask; node i is written at cache
position start + i with RoPE position start + depth(i); the logits of every node go to the
on-device verifier (tree_verify in spec.cu: greedy or multi-draft rejection sampling), and
only (accepted path, final token) returns to the host. Rejected nodes are rolled back by
truncating ``num_computed``; an accepted branch that is not the index-ordered chain is
compacted to contiguous positions by kv_compact.

Proposers (the reference's speculative/ package):
  * prompt lookup (squish/speculative/prompt_lookup.py:96-182, prompt_lookup_batched.py) —
    n-gram matches in the request's own tokens, several distinct continuations become
    branches of one tree; lossless (deterministic drafts); an adaptive guard pauses a
    request's drafting after repeated misses (prompt_lookup_batched.py:32-65);
  * draft model (speculative/speculative.py:614-1057) — a small model of the same
    vocabulary proposes k tokens per round from its own paged KV cache, batched over all
    requests; its softmax rows are the q of the rejection test;
  * Jacobi (experimental/jacobi_decode.py:184-330) — the previous verification's own
    predictions past the accepted point are the next guess (fixed-point iteration);
  * Medusa heads (speculative/speculative.py:1821-2050) — extra heads on the final hidden
    state propose the tokens after the next one; the best rank paths of their top-k lists
    form the tree (engine/medusa.py);
  * EAGLE draft head (speculative/speculative.py:416-580) — a one-layer draft model over the
    target's features and token embeddings proposes a greedy chain (engine/eagle.py).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

MAX_TREE_NODES = 32
TREE_META_INTS = 2 + 3 * MAX_TREE_NODES


@dataclass
class SpecConfig:
    method: str = "prompt_lookup"   # prompt_lookup | draft | jacobi | medusa | eagle | redrafter
    k: int = 4                      # draft depth (tokens per branch)
    branches: int = 1               # prompt lookup: distinct continuations per tree
    max_nodes: int = 16             # tree size cap (<= 32)
    ngram_max: int = 3
    ngram_min: int = 1
    draft_model: str | None = None  # preset name or checkpoint path (method "draft")
    adaptive: bool = True           # pause drafting for a request after repeated misses
    miss_limit: int = 4
    cooldown: int = 8
    force_accept: int | None = None  # benchmark knob: accept exactly this many drafts (0..k)
    # Medusa heads (method "medusa"): a head file / directory, or "random:<num_heads>" (tests,
    # benchmarks); candidates per head; paths kept from the Cartesian product
    medusa_heads: str | None = None
    medusa_top_k: int = 4
    medusa_paths: int = 16
    # EAGLE draft head (method "eagle") / recurrent drafter (method "redrafter"): a head file or
    # directory, or "random" (tests, benchmarks)
    eagle_head: str | None = None
    redrafter_head: str | None = None


@dataclass
class DraftTree:
    tokens: list[int]
    parent: list[int]
    qrow: list[int]
    depth: list[int] = field(default_factory=list)

    def __post_init__(self):
        if not self.depth:
            d = [0] * len(self.tokens)
            for i in range(1, len(self.tokens)):
                d[i] = d[self.parent[i]] + 1
            self.depth = d

    @property
    def size(self) -> int:
        return len(self.tokens)

    def masks(self) -> list[int]:
        """Ancestor bitmask (self included) of every node, as int32 values."""
        m = [0] * self.size
        for i in range(self.size):
            v = 1 << i
            if i:
                v |= m[self.parent[i]]
            m[i] = v
        return [x - (1 << 32) if x >= 1 << 31 else x for x in m]

    def meta_row(self, row0: int) -> np.ndarray:
        out = np.full(TREE_META_INTS, -1, dtype=np.int32)
        n = self.size
        out[0], out[1] = row0, n
        out[2:2 + n] = self.parent
        out[2 + MAX_TREE_NODES:2 + MAX_TREE_NODES + n] = self.tokens
        out[2 + 2 * MAX_TREE_NODES:2 + 2 * MAX_TREE_NODES + n] = self.qrow
        return out


def build_tree(root: int, chains: list[list[int]], max_nodes: int, qrows: list[list[int]] | None = None) -> DraftTree:
    """Merge branch chains (best first) into a prefix tree rooted at ``root``; parents
    precede children and each node's children keep chain priority order."""
    tokens, parent, qrow = [root], [-1], [-1]
    kids: dict[tuple[int, int], int] = {}
    for bi, ch in enumerate(chains):
        u = 0
        for j, t in enumerate(ch):
            key = (u, int(t))
            if key in kids:
                u = kids[key]
                continue
            if len(tokens) >= max_nodes:
                break
            tokens.append(int(t))
            parent.append(u)
            qrow.append(qrows[bi][j] if qrows is not None else -1)
            kids[key] = len(tokens) - 1
            u = len(tokens) - 1
    return DraftTree(tokens, parent, qrow)


# ----------------------------------------------------------------------------- proposers
class _Guard:
    """Adaptive miss guard: after ``limit`` verifications without an accepted draft, skip
    drafting for ``cooldown`` steps (the decode then runs as a plain CUDA-graph step)."""

    def __init__(self, limit: int, cooldown: int):
        self.limit, self.cooldown = limit, cooldown
        self.misses: dict[str, int] = {}
        self.paused: dict[str, int] = {}

    def allow(self, rid: str) -> bool:
        left = self.paused.get(rid, 0)
        if left > 0:
            self.paused[rid] = left - 1
            return False
        return True

    def record(self, rid: str, accepted: int) -> None:
        if accepted > 0:
            self.misses[rid] = 0
            return
        m = self.misses.get(rid, 0) + 1
        self.misses[rid] = m
        if m >= self.limit:
            self.paused[rid] = self.cooldown
            self.misses[rid] = 0

    def forget(self, rid: str) -> None:
        self.misses.pop(rid, None)
        self.paused.pop(rid, None)


class NGramIndex:
    """Positions of every n-gram (n in [n_min, n_max]) of a growing token list."""

    def __init__(self, n_min: int, n_max: int):
        self.n_min, self.n_max = n_min, n_max
        self.maps = {n: {} for n in range(n_min, n_max + 1)}
        self.indexed = 0  # tokens covered (an n-gram ending at position i is indexed once i < indexed)

    def update(self, toks: list[int]) -> None:
        for end in range(self.indexed, len(toks)):
            for n, mp in self.maps.items():
                if end + 1 >= n:
                    mp.setdefault(tuple(toks[end + 1 - n:end + 1]), []).append(end)
        self.indexed = len(toks)

    def continuations(self, toks: list[int], k: int, want: int) -> list[list[int]]:
        """Up to ``want`` distinct continuations of the current suffix, longest match first,
        most recent occurrence first."""
        out: list[list[int]] = []
        seen = set()
        L = len(toks)
        for n in range(self.n_max, self.n_min - 1, -1):
            if L < n + 1:
                continue
            ends = self.maps[n].get(tuple(toks[L - n:]), [])
            for end in reversed(ends):
                if end >= L - 1:
                    continue  # the suffix itself
                cont = toks[end + 1:end + 1 + k]
                if not cont:
                    continue
                key = tuple(cont)
                if key in seen:
                    continue
                seen.add(key)
                out.append(cont)
                if len(out) >= want:
                    return out
            if out:
                return out
        return out


class PromptLookupProposer:
    deterministic = True

    def __init__(self, sc: SpecConfig):
        self.sc = sc
        self.index: dict[str, NGramIndex] = {}

    def propose(self, reqs) -> dict[str, DraftTree]:
        """Drafts from the C++ n-gram index (``_C.host.NGramIndex``), fed only the tokens each
        request gained since its last proposal."""
        from .._ext import native

        trees = {}
        for r in reqs:
            idx = self.index.get(r.rid)
            if idx is None:
                idx = self.index[r.rid] = native().host.NGramIndex(self.sc.ngram_min, self.sc.ngram_max)
            have, total = len(idx), r.total_len
            if total > have:
                idx.extend(r.token_slice(have, total - have))
            chains = idx.continuations(self.sc.k, self.sc.branches)
            if chains:
                trees[r.rid] = build_tree(r.token_at(total - 1), chains, self.sc.max_nodes)
        return trees

    def after_verify(self, r, accepted: int, preds=None) -> None:
        pass

    def forget(self, rid: str) -> None:
        self.index.pop(rid, None)


class JacobiProposer:
    """Guess k future tokens; the verification's per-node greedy predictions past the
    accepted point become the next guess. The first guess comes from prompt lookup, else
    repeats the last token."""
    deterministic = True
    wants_preds = True

    def __init__(self, sc: SpecConfig):
        self.sc = sc
        self.guess: dict[str, list[int]] = {}
        self.lookup = PromptLookupProposer(SpecConfig(k=sc.k, branches=1, ngram_max=sc.ngram_max,
                                                      ngram_min=sc.ngram_min))

    def propose(self, reqs) -> dict[str, DraftTree]:
        trees = {}
        for r in reqs:
            g = self.guess.pop(r.rid, None)
            if not g:
                t = self.lookup.propose([r]).get(r.rid)
                g = t.tokens[1:] if t else [r.tokens[-1]] * self.sc.k
            g = g[: self.sc.k]
            if len(g) < self.sc.k:
                g = g + [g[-1]] * (self.sc.k - len(g))
            trees[r.rid] = build_tree(r.tokens[-1], [g], self.sc.max_nodes)
        return trees

    def after_verify(self, r, accepted: int, preds=None) -> None:
        # preds[i] = target greedy token after node i of the chain; nodes accepted+1.. are
        # conditioned on guesses, which is exactly the Jacobi update
        if preds is not None and len(preds) > accepted + 1:
            self.guess[r.rid] = [int(x) for x in preds[accepted + 1:]]

    def forget(self, rid: str) -> None:
        self.guess.pop(rid, None)
        self.lookup.forget(rid)


class DraftModelProposer:
    """A small model proposes a k-token chain per request from its own paged KV cache."""
    deterministic = False

    def __init__(self, sc: SpecConfig, target, draft_engine):
        from .request import Request

        self.sc = sc
        self.target = target
        self.eng = draft_engine
        self._Request = Request
        self.seqs: dict[str, object] = {}
        import torch

        V = target.cfg.vocab_size
        self.vd = draft_engine.cfg.vocab_size
        if self.vd > V:
            raise ValueError(f"draft vocabulary {self.vd} exceeds the target vocabulary {V}")
        dev = getattr(draft_engine.runner, "device", torch.device("cpu"))
        # q rows over the target vocabulary; ids the draft cannot emit keep q = 0 (logit -inf)
        self.qbuf = torch.full((target.ecfg.max_num_seqs * sc.k, V), float("-inf"), dtype=torch.bfloat16, device=dev)

    def _seq(self, r):
        s = self.seqs.get(r.rid)
        if s is None:
            from .sampling import SamplingParams

            s = self._Request(r.rid, list(r.tokens), SamplingParams(max_tokens=1 << 30, ignore_eos=True,
                                                                   temperature=r.params.temperature))
            self.seqs[r.rid] = s
        return s

    def propose(self, reqs) -> dict[str, DraftTree]:
        import torch

        from .scheduler import ScheduledEntry

        sc, eng = self.sc, self.eng
        reqs = [r for r in reqs if len(r.tokens) + sc.k < eng.ecfg.max_model_len]
        if not reqs:
            return {}
        seqs = []
        for r in reqs:
            s = self._seq(r)
            keep = min(s.num_computed, len(r.tokens) - 1)
            # the draft KV is valid for the common prefix of what it computed and the target tokens
            common = 0
            old = s.tokens
            new = [t if t < self.vd else 0 for t in r.tokens]
            for a, b in zip(old[:keep], new[:keep]):
                if a != b:
                    break
                common += 1
            # ids the draft's vocabulary lacks (the target's may be larger) become id 0 there
            s.prompt = [t if t < self.vd else 0 for t in r.tokens]
            s.output = []
            s.num_computed = common
            s.params.temperature = r.params.temperature
            seqs.append(s)
        drafts = [[] for _ in seqs]
        qrows = [[] for _ in seqs]
        for j in range(sc.k):
            dec, pre = [], []
            for s in seqs:
                n = s.total_len - s.num_computed
                if not eng.scheduler._ensure_pages(s, s.total_len):
                    return {}
                e = ScheduledEntry(s, s.num_computed, n, True)
                (dec if n == 1 and s.num_computed > 0 else pre).append(e)
            order = dec + pre
            toks = eng.run_entries(dec, pre)
            logits = eng.runner.logits
            for i, e in enumerate(order):
                si = seqs.index(e.req)
                row = si * sc.k + j
                self.qbuf[row, : self.vd].copy_(logits[i, : self.vd])
                drafts[si].append(int(toks[i]))
                qrows[si].append(row)
                e.req.num_computed = e.start + e.n
                e.req.output.append(int(toks[i]))
                e.req.rng_step += 1
        if isinstance(self.qbuf, torch.Tensor) and self.qbuf.is_cuda:
            torch.cuda.current_stream(self.qbuf.device).synchronize()
        return {r.rid: build_tree(r.tokens[-1], [drafts[i]], sc.max_nodes, [qrows[i]]) for i, r in enumerate(reqs)}

    def after_verify(self, r, accepted: int, preds=None) -> None:
        s = self.seqs.get(r.rid)
        if s is not None:
            # draft KV stays valid up to the last accepted draft token
            s.num_computed = min(s.num_computed, len(r.tokens) - 1)

    def forget(self, rid: str) -> None:
        s = self.seqs.pop(rid, None)
        if s is not None:
            self.eng.scheduler.blocks.release(s.pages)
            s.pages = []


class MedusaProposer:
    """Drafts from Medusa heads (engine/medusa.py) over the final hidden state of the row that
    produced each request's newest token: the engine calls ``observe`` after every step with
    those rows; ``propose`` turns a request's per-head top-k lists into a tree of the best rank
    paths rooted at the pending token."""
    deterministic = True
    wants_hidden = True

    def __init__(self, sc: SpecConfig, heads):
        self.sc = sc
        self.heads = heads
        self.cands: dict[str, np.ndarray] = {}

    def observe(self, reqs, hidden) -> None:
        if not reqs:
            return
        tops = self.heads.topk(hidden, self.sc.medusa_top_k)
        for r, t in zip(reqs, tops):
            self.cands[r.rid] = t

    def propose(self, reqs) -> dict[str, DraftTree]:
        from .medusa import rank_paths

        trees = {}
        n, k = self.heads.num_heads, self.sc.medusa_top_k
        depth = min(n, self.sc.k)
        paths = rank_paths(depth, k, self.sc.medusa_paths)
        for r in reqs:
            c = self.cands.pop(r.rid, None)
            if c is None:
                continue
            chains = [[int(c[h, rk]) for h, rk in enumerate(p)] for p in paths]
            trees[r.rid] = build_tree(r.token_at(r.total_len - 1), chains, self.sc.max_nodes)
        return trees

    def after_verify(self, r, accepted: int, preds=None) -> None:
        pass

    def forget(self, rid: str) -> None:
        self.cands.pop(rid, None)


class EagleProposer:
    """Drafts from an EAGLE head (engine/eagle.py): ``observe`` commits each live request's
    (feature, newest token) pair to its head history and keeps the resulting position;
    ``propose`` drafts k greedy tokens from it for all requests in one batch per draft step."""
    deterministic = True
    wants_hidden = True

    def __init__(self, sc: SpecConfig, head):
        self.sc = sc
        self.head = head
        self.states: dict[str, dict] = {}
        self.start: dict[str, tuple] = {}

    def observe(self, reqs, hidden) -> None:
        if not reqs:
            return
        states = [self.states.setdefault(r.rid, self.head.new_state()) for r in reqs]
        toks = [r.token_at(r.total_len - 1) for r in reqs]
        h, logits = self.head.step(states, hidden, toks, commit=True)
        for i, r in enumerate(reqs):
            self.start[r.rid] = (h[i], logits[i])

    def propose(self, reqs) -> dict[str, DraftTree]:
        import torch

        reqs = [r for r in reqs if r.rid in self.start]
        if not reqs:
            return {}
        starts = [self.start.pop(r.rid) for r in reqs]
        h = torch.stack([s[0] for s in starts])
        logits = torch.stack([s[1] for s in starts])
        drafts = self.head.draft([self.states[r.rid] for r in reqs], h, logits, self.sc.k)
        return {r.rid: build_tree(r.token_at(r.total_len - 1), [d], self.sc.max_nodes) for r, d in zip(reqs, drafts)}

    def after_verify(self, r, accepted: int, preds=None) -> None:
        pass

    def forget(self, rid: str) -> None:
        self.states.pop(rid, None)
        self.start.pop(rid, None)


class ReDrafterProposer:
    """Drafts from a recurrent drafter (engine/redrafter.py): the feature that produced each
    request's newest token starts the GRU; greedy chains batched over requests."""
    deterministic = True
    wants_hidden = True

    def __init__(self, sc: SpecConfig, head):
        self.sc = sc
        self.head = head
        self.feat: dict[str, object] = {}

    def observe(self, reqs, hidden) -> None:
        for r, f in zip(reqs, hidden):
            self.feat[r.rid] = f

    def propose(self, reqs) -> dict[str, DraftTree]:
        import torch

        reqs = [r for r in reqs if r.rid in self.feat]
        if not reqs:
            return {}
        feats = torch.stack([self.feat.pop(r.rid) for r in reqs])
        toks = [r.token_at(r.total_len - 1) for r in reqs]
        drafts = self.head.draft(feats, toks, self.sc.k)
        return {r.rid: build_tree(t, [d], self.sc.max_nodes) for r, t, d in zip(reqs, toks, drafts)}

    def after_verify(self, r, accepted: int, preds=None) -> None:
        pass

    def forget(self, rid: str) -> None:
        self.feat.pop(rid, None)


def _tied_tensors(target):
    ck = getattr(target, "checkpoint_tensors", None)
    if ck is None:
        raise ValueError("a feature-based drafter needs the target checkpoint's embedding, final norm and LM head")
    emb = ck["model.embed_tokens.weight"].dequantize()
    lm = ck["lm_head.weight"].dequantize() if "lm_head.weight" in ck else emb
    return emb, lm, ck["model.norm.weight"].dequantize()


def load_redrafter_head(sc: SpecConfig, target):
    from .redrafter import ReDrafterHead

    emb, lm, norm = _tied_tensors(target)
    dev = getattr(target.runner, "device", "cpu")
    spec = sc.redrafter_head or "random"
    if spec == "random":
        return ReDrafterHead.random(target.cfg, emb, lm, norm, device=dev)
    return ReDrafterHead.load(spec, target.cfg, emb, lm, norm, device=dev)


def load_eagle_head(sc: SpecConfig, target):
    """The EAGLE head on the target's device, tied to the target's embedding, final norm and
    LM head (dequantized to fp32 once)."""
    from .eagle import EagleHead

    cfg = target.cfg
    dev = getattr(target.runner, "device", "cpu")
    ck = getattr(target, "checkpoint_tensors", None)
    if ck is None:
        raise ValueError("the EAGLE head needs the target checkpoint's embedding, final norm and LM head")
    emb = ck["model.embed_tokens.weight"].dequantize()
    lm = ck["lm_head.weight"].dequantize() if "lm_head.weight" in ck else emb
    norm = ck["model.norm.weight"].dequantize()
    spec = sc.eagle_head or "random"
    if spec == "random":
        return EagleHead.random(cfg, emb, lm, norm, device=dev)
    return EagleHead.load(spec, cfg, emb, lm, norm, device=dev)


def load_medusa_heads(sc: SpecConfig, target):
    """The proposer's heads on the target's device: a file / directory, or random heads."""
    from .medusa import MedusaHeads

    cfg = target.cfg
    dev = getattr(target.runner, "device", "cpu")
    spec = sc.medusa_heads or "random:3"
    if spec.startswith("random"):
        n = int(spec.split(":", 1)[1]) if ":" in spec else 3
        return MedusaHeads.random(cfg.hidden_size, cfg.vocab_size, num_heads=n, device=dev)
    heads = MedusaHeads.load(spec, device=dev)
    if heads.hidden != cfg.hidden_size or heads.vocab != cfg.vocab_size:
        raise ValueError(f"Medusa heads are {heads.hidden} -> {heads.vocab}; the model is "
                         f"{cfg.hidden_size} -> {cfg.vocab_size}")
    return heads


def make_proposer(sc: SpecConfig, target):
    if sc.method == "prompt_lookup":
        return PromptLookupProposer(sc)
    if sc.method == "jacobi":
        return JacobiProposer(sc)
    if sc.method == "medusa":
        return MedusaProposer(sc, load_medusa_heads(sc, target))
    if sc.method == "eagle":
        return EagleProposer(sc, load_eagle_head(sc, target))
    if sc.method == "redrafter":
        return ReDrafterProposer(sc, load_redrafter_head(sc, target))
    if sc.method == "draft":
        if not sc.draft_model:
            raise ValueError("speculative method 'draft' needs draft_model")
        from ..api import load_engine
        from .engine import EngineConfig

        dev = getattr(target.runner, "device", "cpu")
        te = target.ecfg
        pages = te.max_num_seqs * ((te.max_model_len + 15) // 16 + 2)
        de = load_engine(sc.draft_model, str(dev), kv_dtype=target.qcfg.kv_dtype,
                         ecfg=EngineConfig(max_num_seqs=te.max_num_seqs, max_num_batched_tokens=te.max_num_batched_tokens,
                                           max_model_len=te.max_model_len, num_pages=pages,
                                           enable_prefix_caching=False, cuda_graphs=te.cuda_graphs)).engine
        return DraftModelProposer(sc, target, de)
    raise ValueError(f"unknown speculative method {sc.method!r}")


def spec_eligible(params) -> bool:
    """Requests whose sampling the verifier reproduces exactly: greedy, or temperature-only
    sampling (no top-k/top-p/min-p, repetition penalty or grammar)."""
    return (params.grammar is None and params.repetition_penalty == 1.0 and params.top_k == 0
            and params.top_p >= 1.0 and params.min_p <= 0.0 and not params.logprobs)


# ----------------------------------------------------------------------------- host oracle
_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _mix64(z: np.ndarray) -> np.ndarray:
    z = z + np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def _uni(seed: int, a: int, b: int, c) -> np.ndarray:
    """The verifier's counter-hash uniforms in (0, 1), bit-identical to the device draw."""
    with np.errstate(over="ignore"):
        c = np.asarray(c, dtype=np.uint64)
        inner = _mix64(np.uint64(b) ^ (c << np.uint64(24)))
        h = _mix64(np.uint64(seed) ^ _mix64(np.uint64(a) * np.uint64(0x100000001B3) + inner))
    return ((h >> np.uint64(40)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 16777216.0)


def tree_verify_ref(logits, tree: DraftTree, temperature: float, seed: int, step: int, draft_logits=None):
    """Host restatement of the device verifier: returns (accepted node list, final token)."""
    import torch

    lg = logits.float().cpu().numpy()
    ql = None if draft_logits is None else draft_logits.float().cpu().numpy()
    n = tree.size
    u, path = 0, []
    V = lg.shape[1]
    step = int(step) & 0xFFFFFFFF
    for _ in range(MAX_TREE_NODES + 1):
        kids = [c for c in range(1, n) if tree.parent[c] == u]
        row = lg[u]
        if temperature <= 0:
            am = int(np.argmax(row))
            nxt = next((c for c in kids if tree.tokens[c] == am), -1)
            if nxt < 0:
                return path, am
            path.append(nxt)
            u = nxt
            continue
        z = row / temperature
        p = np.exp(z - z.max())
        p /= p.sum()
        res = None
        nxt = -1
        for c in kids:
            x = tree.tokens[c]
            px = p[x] if res is None else res[x]
            q = None
            qx = 1.0
            if tree.qrow[c] >= 0 and ql is not None:
                zq = ql[tree.qrow[c]] / temperature
                q = np.exp(zq - zq.max())
                q /= q.sum()
                qx = q[x]
            ur = float(_uni(seed, step, u * 64 + c, 0x5EED))
            if ur < min(1.0, px / max(qx, 1e-30)):
                nxt = c
                break
            res = p.copy() if res is None else res
            if q is not None:
                res = np.maximum(0.0, res - q)
            else:
                res[x] = 0.0
            s = res.sum()
            res = res / s if s > 0 else None
        if nxt >= 0:
            path.append(nxt)
            u = nxt
            continue
        g = -np.log(-np.log(_uni(seed, step, 0x10000 + u, np.arange(V))))
        key = np.where(res > 0, np.log(np.maximum(res, 1e-38)) + g, -np.inf) if res is not None else z + g
        return path, int(np.argmax(key))
    return path, 0
