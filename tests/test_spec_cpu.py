"""Speculative decoding on the CPU oracle: draft trees, n-gram lookup, the verifier's host
restatement (greedy exactness and the lossless sampling property), and the engine paths
(prompt lookup with branching trees, Jacobi, draft model, Medusa heads) against plain greedy
decoding.

Mirrors the reference's greedy-identity contract (tests/test_prompt_lookup_batched.py):
speculation must not change greedy output.
"""
import numpy as np
import pytest
import torch

from squish_b200.engine.engine import EngineConfig, LLMEngine
from squish_b200.engine.sampling import SamplingParams
from squish_b200.engine.speculative import (NGramIndex, SpecConfig, _uni, build_tree, tree_verify_ref)
from squish_b200.models.config import get_preset
from squish_b200.models.weights import random_checkpoint


def test_build_tree_merges_prefixes_and_masks():
    t = build_tree(7, [[1, 2, 3], [1, 2, 4], [5]], max_nodes=16)
    assert t.tokens == [7, 1, 2, 3, 4, 5]
    assert t.parent == [-1, 0, 1, 2, 2, 0]
    assert t.depth == [0, 1, 2, 3, 3, 1]
    m = t.masks()
    assert m[3] == 0b001111 and m[4] == 0b010111 and m[5] == 0b100001
    t2 = build_tree(7, [[1, 2, 3], [9, 9, 9]], max_nodes=5)
    assert t2.size == 5 and t2.tokens == [7, 1, 2, 3, 9]


def test_ngram_continuations():
    idx = NGramIndex(1, 3)
    toks = [1, 2, 3, 4, 9, 1, 2, 3, 5, 7, 1, 2, 3]
    idx.update(toks)
    c = idx.continuations(toks, 3, 2)
    assert c == [[5, 7, 1], [4, 9, 1]]  # most recent match of (1,2,3) first
    idx.update(toks + [8])
    assert idx.continuations(toks + [8], 2, 1) == []


def test_uniform_hash_is_in_range_and_deterministic():
    u = _uni(1, 2, 3, np.arange(1000))
    assert (u > 0).all() and (u < 1).all() and abs(float(u.mean()) - 0.5) < 0.05
    assert np.array_equal(u, _uni(1, 2, 3, np.arange(1000)))


def test_verify_ref_greedy_follows_argmax_chain():
    V = 50
    lg = torch.full((5, V), -5.0)
    # root predicts 3; node(3) predicts 8; node(8) predicts 2
    lg[0, 3] = lg[1, 8] = lg[2, 2] = 5.0
    lg[3, 1] = lg[4, 1] = 5.0
    t = build_tree(0, [[3, 8, 9], [4]], 16)  # nodes: 3,8,9 chain then 4
    path, fin = tree_verify_ref(lg, t, 0.0, 0, 0)
    assert path == [1, 2] and fin == 2  # 3 and 8 accepted, 9 rejected -> argmax at node(8) = 2


def test_verify_ref_sampling_is_lossless():
    """First emitted token ~ p whatever the (deterministic or model) draft: chi-square check."""
    V = 6
    g = torch.Generator().manual_seed(0)
    lg = torch.randn(4, V, generator=g) * 1.5
    p = torch.softmax(lg[0], -1).numpy()
    ql = torch.randn(2, V, generator=g)
    N = 4000
    for kind in ("lookup", "draft"):
        counts = np.zeros(V)
        for s in range(N):
            if kind == "lookup":
                t = build_tree(0, [[2, 1], [4]], 16)
                path, fin = tree_verify_ref(lg, t, 1.0, 123, s)
            else:
                q = torch.softmax(ql[0], -1).numpy()
                d1 = int(np.searchsorted(np.cumsum(q), _uni(7, s, 1, 0)))  # draft sample from q
                d1 = min(d1, V - 1)
                t = build_tree(0, [[d1]], 16, [[0]])
                path, fin = tree_verify_ref(lg[:2], t, 1.0, 123, s, draft_logits=ql)
            first = t.tokens[path[0]] if path else fin
            counts[first] += 1
        exp = p * N
        chi2 = float(((counts - exp) ** 2 / exp).sum())
        assert chi2 < 25.0, (kind, chi2, counts, exp)  # 5 dof: p ~ 1e-4


def _engine(spec=None, seed=0):
    cfg, q = get_preset("tiny-llama")
    ck = random_checkpoint(cfg, q, seed=seed, device="cpu")
    return LLMEngine.from_checkpoint(ck, "cpu", EngineConfig(max_num_seqs=4, max_num_batched_tokens=256,
                                                             max_model_len=512, num_pages=128, cuda_graphs=False,
                                                             spec=spec))


def _prompts():
    rng = np.random.default_rng(3)
    base = rng.integers(0, 32000, 12).tolist()
    return [base * 3 + base[:5], rng.integers(0, 32000, 20).tolist() * 2]


@pytest.mark.parametrize("spec", [SpecConfig("prompt_lookup", k=4, branches=3, max_nodes=12),
                                  SpecConfig("jacobi", k=3), SpecConfig("draft", k=3, draft_model="tiny-llama"),
                                  SpecConfig("medusa", k=3, medusa_heads="random:3", medusa_top_k=2),
                                  SpecConfig("eagle", k=3, eagle_head="random"),
                                  SpecConfig("redrafter", k=3, redrafter_head="random")])
def test_speculative_greedy_matches_plain_greedy(spec):
    sp = SamplingParams(max_tokens=24, ignore_eos=True)
    want = _engine().generate(_prompts(), sp)
    eng = _engine(spec)
    got = eng.generate(_prompts(), sp)
    assert got == want
    st = eng.spec_stats
    assert st["verifies"] > 0 and st["emitted"] >= st["verifies"]
    if spec.method == "draft":  # the draft is the target itself: every draft is accepted
        assert st["accepted"] == st["drafted"]


def test_force_accept_knob_emits_fixed_lengths():
    sc = SpecConfig("jacobi", k=4, force_accept=2, adaptive=False)
    eng = _engine(sc)
    out = eng.generate([_prompts()[0]], SamplingParams(max_tokens=13, ignore_eos=True))[0]
    assert len(out) == 13
    assert eng.spec_stats["accepted"] == 2 * eng.spec_stats["verifies"]


def test_second_branch_acceptance_compacts_kv():
    """A tree whose first branch is wrong and second branch is the true continuation: the
    accepted nodes are not the index-ordered chain, so their KV rows must be moved."""
    prompt = _prompts()[1]
    sp = SamplingParams(max_tokens=12, ignore_eos=True)
    want = _engine().generate([prompt], sp)[0]
    eng = _engine(SpecConfig("prompt_lookup", k=3, branches=2, max_nodes=16, adaptive=False))

    class Oracle:
        def propose(self, reqs):
            out = {}
            for r in reqs:
                done = len(r.output)
                true = want[done:done + 3]
                wrong = [(t + 1) % 32000 for t in true]
                if true:
                    out[r.rid] = build_tree(r.tokens[-1], [wrong, true], 16)
            return out

        def after_verify(self, r, accepted, preds=None):
            pass

        def forget(self, rid):
            pass

    eng.proposer = Oracle()
    calls = []
    orig = eng.runner.kv_compact
    eng.runner.kv_compact = lambda s, d: (calls.append((list(s), list(d))), orig(s, d))
    got = eng.generate([prompt], sp)[0]
    assert got == want
    assert calls, "the second branch should have been compacted"
    assert eng.spec_stats["accepted"] > 0


def test_cpp_ngram_index_matches_python():
    """The C++ prompt-lookup index gives the same continuations as the Python restatement,
    fed incrementally."""
    import numpy as np

    from squish_b200._ext import native
    from squish_b200.engine.speculative import NGramIndex

    rng = np.random.default_rng(0)
    for trial in range(20):
        base = rng.integers(0, 12 if trial % 2 else 400, 300).tolist()
        toks = base + base[50:90] + rng.integers(0, 12, 30).tolist()
        py = NGramIndex(1, 4)
        cc = native().host.NGramIndex(1, 4)
        pos = 0
        for cut in sorted(rng.integers(5, len(toks), 6).tolist()) + [len(toks)]:
            cc.extend(toks[pos:cut])
            pos = max(pos, cut)
            py.update(toks[:pos])
            assert len(cc) == pos
            for k, want in ((4, 1), (6, 3)):
                assert cc.continuations(k, want) == py.continuations(toks[:pos], k, want)


def test_medusa_heads_roundtrip_and_rank_paths(tmp_path):
    from safetensors.torch import save_file

    from squish_b200.engine.medusa import MedusaHeads, rank_paths

    heads = MedusaHeads.random(64, 300, num_heads=3, num_layers=1, seed=1)
    sd = heads.state_dict()
    assert sorted(sd) == sorted([f"medusa_head.{i}.0.linear.{n}" for i in range(3) for n in ("weight", "bias")] +
                                [f"medusa_head.{i}.1.weight" for i in range(3)])
    save_file(sd, str(tmp_path / "medusa_lm_head.safetensors"))
    back = MedusaHeads.load(tmp_path)
    h = torch.randn(5, 64)
    for a, b in zip(heads.logits(h), back.logits(h)):
        torch.testing.assert_close(a, b)
    # the reference's plain linear head (no residual block, a bias)
    lin = {"medusa_head.0.0.weight": torch.randn(300, 64), "medusa_head.0.0.bias": torch.randn(300)}
    one = MedusaHeads.from_state_dict(lin)
    want = h @ lin["medusa_head.0.0.weight"].T + lin["medusa_head.0.0.bias"]
    torch.testing.assert_close(one.logits(h)[0], want)
    assert one.topk(h, 3).shape == (5, 1, 3)
    assert np.array_equal(one.topk(h, 3)[:, 0], want.topk(3, -1).indices.numpy())
    p = rank_paths(3, 2, 5)
    assert p[0] == (0, 0, 0) and sorted(p[1:4]) == [(0, 0, 1), (0, 1, 0), (1, 0, 0)] and sum(p[4]) == 2


def test_medusa_sees_the_rows_that_produced_each_token():
    """The Medusa proposer gets, after every step, the final-norm hidden row whose logits gave
    each request's newest token (decode rows and the last accepted node of a verified tree);
    with oracle candidates (the true continuation at rank 1) drafts are accepted and greedy
    output is unchanged."""
    prompt = _prompts()[1]
    sp = SamplingParams(max_tokens=16, ignore_eos=True)
    want = _engine().generate([prompt], sp)[0]
    eng = _engine(SpecConfig("medusa", k=3, medusa_heads="random:3", medusa_top_k=2, medusa_paths=8,
                             max_nodes=16, adaptive=False))
    prop = eng.proposer
    lm = eng.runner.ref.w["lm_head.weight"].float()
    seen = []

    def observe(reqs, hidden):
        for r, h in zip(reqs, hidden):
            seen.append(int((h.float() @ lm.T).argmax()) == r.output[-1])
            done = len(r.output)
            true = (want[done:done + 3] + [0, 0, 0])[:3]
            cand = np.zeros((3, 2), dtype=np.int32)
            cand[:, 0] = [(t + 1) % 32000 for t in true]
            cand[:, 1] = true
            prop.cands[r.rid] = cand

    prop.observe = observe
    got = eng.generate([prompt], sp)[0]
    assert got == want
    assert seen and all(seen), seen
    assert eng.spec_stats["accepted"] > 0


def test_eagle_head_batched_step_matches_a_full_causal_pass(tmp_path):
    """The head's incremental, batched steps equal one causal pass of its decoder layer over the
    same (feature, token) sequence, and the published tensor names round-trip."""
    import math

    from safetensors.torch import save_file

    from squish_b200.engine.eagle import EagleHead
    from squish_b200.models.reference import _rms, _rope, rope_table

    cfg, _ = get_preset("tiny-llama")
    g = torch.Generator().manual_seed(0)
    emb = torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g)
    lm = torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g) * 0.05
    head = EagleHead.random(cfg, emb, lm, torch.ones(cfg.hidden_size), seed=3)
    T = 6
    feats = torch.randn(2, T, cfg.hidden_size, generator=g)
    toks = torch.randint(0, cfg.vocab_size, (2, T), generator=g)
    states = [head.new_state(), head.new_state()]
    got = [head.step(states, feats[:, t], toks[:, t].tolist(), commit=True)[0] for t in range(T)]
    got = torch.stack(got, 1)  # [2, T, H]
    t_, d, hq, hkv = head.t, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    for b in range(2):
        z = torch.cat([feats[b], emb[toks[b]]], 1) @ t_["fc.weight"].T + t_["fc.bias"]
        cs = rope_table(cfg, T)
        q = _rope((z @ t_["layers.0.self_attn.q_proj.weight"].T).view(T, hq, d), cs)
        k = _rope((z @ t_["layers.0.self_attn.k_proj.weight"].T).view(T, hkv, d), cs).repeat_interleave(hq // hkv, 1)
        v = (z @ t_["layers.0.self_attn.v_proj.weight"].T).view(T, hkv, d).repeat_interleave(hq // hkv, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(d)
        s = s.masked_fill(torch.ones(T, T).triu(1).bool(), float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(T, -1)
        h = z + o @ t_["layers.0.self_attn.o_proj.weight"].T
        m = _rms(h, t_["layers.0.post_attention_layernorm.weight"], cfg.rms_eps)
        h = h + (torch.nn.functional.silu(m @ t_["layers.0.mlp.gate_proj.weight"].T)
                 * (m @ t_["layers.0.mlp.up_proj.weight"].T)) @ t_["layers.0.mlp.down_proj.weight"].T
        torch.testing.assert_close(got[b], h, rtol=1e-4, atol=1e-4)
    # drafting leaves the committed history as it was
    n0 = states[0]["k"].shape[0]
    h0, lg = head.step(states, feats[:, 0], [1, 2], commit=True)
    head.draft(states, h0, lg, 4)
    assert states[0]["k"].shape[0] == n0 + 1
    save_file({"model." + k: v for k, v in head.state_dict().items()}, str(tmp_path / "eagle.safetensors"))
    back = EagleHead.load(tmp_path, cfg, emb, lm, torch.ones(cfg.hidden_size))
    assert all(torch.equal(back.t[k], v) for k, v in head.t.items())


def test_redrafter_gru_matches_torch_cell():
    """The drafter's GRU cell (C++ kernel on the CPU path) equals torch's GRUCell with the same
    weights, and the greedy chain follows its own argmax."""
    from squish_b200.engine.redrafter import ReDrafterHead

    cfg, _ = get_preset("tiny-llama")
    g = torch.Generator().manual_seed(1)
    H = cfg.hidden_size
    emb = torch.randn(cfg.vocab_size, H, generator=g)
    head = ReDrafterHead.random(cfg, emb, torch.randn(cfg.vocab_size, H, generator=g) * 0.05, torch.ones(H), seed=2)
    cell = torch.nn.GRUCell(H, H)
    with torch.no_grad():
        cell.weight_ih.copy_(head.t["gru.weight_ih"])
        cell.weight_hh.copy_(head.t["gru.weight_hh"])
        cell.bias_ih.copy_(head.t["gru.bias_ih"])
        cell.bias_hh.copy_(head.t["gru.bias_hh"])
        e, s = torch.randn(3, H, generator=g), torch.randn(3, H, generator=g)
        torch.testing.assert_close(head.gru(e, s), cell(e, s), rtol=1e-4, atol=1e-5)
    d = head.draft(torch.randn(2, H, generator=g), [5, 9], 4)
    assert [len(x) for x in d] == [4, 4]
