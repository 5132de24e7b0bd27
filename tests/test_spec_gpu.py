"""Speculative decoding kernels on the GPU: tree verification against its host restatement,
tree-masked prefill attention against an fp32 reference, KV compaction, and the engine's
speculative paths against the CPU fp32 oracle."""
import numpy as np
import pytest
import torch

from squish_b200 import ops
from squish_b200.engine.engine import EngineConfig, LLMEngine
from squish_b200.engine.sampling import SamplingParams
from squish_b200.engine.speculative import SpecConfig, build_tree, tree_verify_ref
from squish_b200.models.config import get_preset
from squish_b200.models.reference import ReferenceModel
from squish_b200.models.weights import random_checkpoint

from ._refs import sm_scale
from .test_engine_gpu import _teacher_forced_ok
from .test_kernels_gpu import _fill_random_cache, _gather

pytestmark = pytest.mark.gpu


def _trees(rng, V, G):
    out = []
    for _ in range(G):
        chains = [rng.integers(0, V, int(rng.integers(1, 5))).tolist() for _ in range(int(rng.integers(1, 4)))]
        out.append(build_tree(int(rng.integers(0, V)), chains, 16))
    return out


@pytest.mark.parametrize("temp", [0.0, 0.8])
@pytest.mark.parametrize("with_draft", [False, True])
def test_tree_verify_matches_host(cuda, temp, with_draft):
    if with_draft and temp == 0.0:
        pytest.skip("greedy ignores the draft distribution")
    V, G = 2000, 48
    rng = np.random.default_rng(11)
    trees = _trees(rng, V, G)
    rows = sum(t.size for t in trees)
    g = torch.Generator().manual_seed(1)
    logits = (torch.randn(rows, V, generator=g) * 2).to(torch.bfloat16)
    # make greedy walks non-trivial: each node's argmax is its first child's token half of the time
    r0 = 0
    metas = []
    qrows = 0
    for t in trees:
        for u in range(t.size):
            kids = [c for c in range(1, t.size) if t.parent[c] == u]
            if kids and rng.random() < 0.6:
                logits[r0 + u, t.tokens[kids[int(rng.integers(0, len(kids)))]]] = 12.0
        if with_draft:
            t.qrow = [-1] + list(range(qrows, qrows + t.size - 1))
            qrows += t.size - 1
        metas.append(t.meta_row(r0))
        r0 += t.size
    draft = (torch.randn(max(qrows, 1), V, generator=g) * 2).to(torch.bfloat16) if with_draft else None
    meta = torch.from_numpy(np.stack(metas)).to(cuda)
    temps = torch.full((G,), temp, dtype=torch.float32, device=cuda)
    steps = torch.arange(G, dtype=torch.int32, device=cuda) * 7
    out = torch.zeros(G, 34, dtype=torch.int32, device=cuda)
    ops.kernels.tree_verify(logits.to(cuda), meta, temps, steps, 99, out,
                            draft_logits=draft.to(cuda) if draft is not None else None)
    out = out.cpu()
    agree = 0
    r0 = 0
    for i, t in enumerate(trees):
        path, fin = tree_verify_ref(logits[r0:r0 + t.size], t, temp, 99, int(steps[i]), draft)
        got_path = out[i, 2:2 + int(out[i, 0])].tolist()
        # the node walk must be a valid root-to-node chain
        u = 0
        for c in got_path:
            assert t.parent[c] == u
            u = c
        agree += int(got_path == path and int(out[i, 1]) == fin)
        r0 += t.size
    # greedy is exact; sampled draws use the same hash, so only float rounding at a boundary may differ
    assert agree == G if temp == 0.0 else agree >= G - 2, agree


def test_tree_mask_prefill_attention(cuda):
    ps, group, hq, hkv, d = 16, 32, 8, 2, 128
    fk, fv = ops.KV_FORMATS["int4"]
    tree = build_tree(5, [[1, 2, 3], [1, 4], [6, 7]], 16)  # 7 nodes
    n = tree.size
    ctx_before = 37
    ctx = ctx_before + n
    npg = (ctx + ps - 1) // ps
    kc, ks, vc, vs, kd, vd = _fill_random_cache(npg + 2, hkv, ps, d, fk, fv, group, cuda, seed=5)
    bt = torch.arange(npg, dtype=torch.int32).view(1, -1)
    q = torch.randn(n, hq * d).to(torch.bfloat16)
    out = torch.zeros(n, hq * d, dtype=torch.bfloat16, device=cuda)
    masks = torch.tensor(tree.masks(), dtype=torch.int32)
    i32 = dict(dtype=torch.int32, device=cuda)
    ops.paged_prefill_attention(q.to(cuda), kc, ks, vc, vs, bt.to(cuda), torch.zeros(1, **i32), torch.zeros(1, **i32),
                                torch.zeros(1, **i32), torch.tensor([n], **i32), torch.tensor([ctx], **i32), 1, out,
                                hq, hkv, d, ps, group, fk, fv, sm_scale(d), tree_mask=masks.to(cuda))
    torch.cuda.synchronize()
    k = _gather(kd, bt[0], ctx, ps).to(torch.bfloat16).float()
    v = _gather(vd, bt[0], ctx, ps).to(torch.bfloat16).float()
    kk, vv = k.repeat_interleave(hq // hkv, 1), v.repeat_interleave(hq // hkv, 1)
    s = torch.einsum("qhd,khd->hqk", q.float().view(n, hq, d), kk) * sm_scale(d)
    allow = torch.zeros(n, ctx, dtype=torch.bool)
    allow[:, :ctx_before] = True
    for i in range(n):
        for j in range(n):
            allow[i, ctx_before + j] = bool((int(masks[i]) >> j) & 1)
    s = s.masked_fill(~allow[None], float("-inf"))
    ref = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv)
    torch.testing.assert_close(out.float().cpu().view(n, hq, d), ref, rtol=2e-2, atol=5e-2)


def test_kv_compact_moves_rows(cuda):
    cfg, q = get_preset("tiny-llama")
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0), cuda,
                                    EngineConfig(max_num_seqs=2, max_model_len=256, num_pages=16, cuda_graphs=False))
    pools = eng.runner.pools.layers
    for t in [x for layer in pools for x in layer]:
        t.copy_(torch.randint(0, 255, t.shape, dtype=torch.uint8).view(t.dtype) if t.dtype == torch.uint8
                else torch.randn(t.shape, dtype=torch.float32).to(t.dtype))
    before = [[x.clone() for x in layer] for layer in pools]
    src, dst = [37, 40, 41], [34, 35, 36]
    eng.runner.kv_compact(src, dst)
    torch.cuda.synchronize()
    ps = q.page_size
    for li, layer in enumerate(pools):
        for ti, x in enumerate(layer):
            want = before[li][ti].clone()
            for a, b in zip(src, dst):
                want[b // ps, :, b % ps] = want[a // ps, :, a % ps]
            assert torch.equal(x, want), (li, ti)


@pytest.mark.parametrize("spec", [SpecConfig("prompt_lookup", k=4, branches=3, max_nodes=12),
                                  SpecConfig("jacobi", k=3), SpecConfig("draft", k=3, draft_model="tiny-llama"),
                                  SpecConfig("medusa", k=3, medusa_heads="random:3", medusa_top_k=2)])
def test_speculative_engine_matches_oracle(cuda, spec):
    cfg, q = get_preset("tiny-llama")
    rng = np.random.default_rng(3)
    base = rng.integers(0, cfg.vocab_size, 12).tolist()
    prompts = [base * 3 + base[:5], rng.integers(0, cfg.vocab_size, 20).tolist() * 2]
    eng = LLMEngine.from_checkpoint(random_checkpoint(cfg, q, seed=0), cuda,
                                    EngineConfig(max_num_seqs=4, max_num_batched_tokens=256, max_model_len=512,
                                                 num_pages=128, spec=spec))
    outs = eng.generate(prompts, SamplingParams(max_tokens=24, ignore_eos=True))
    ref = ReferenceModel(random_checkpoint(cfg, q, seed=0))
    for p, o in zip(prompts, outs):
        assert len(o) == 24
        ok, worst = _teacher_forced_ok(ref, p, o)
        assert ok, (worst, o)
    assert eng.spec_stats["verifies"] > 0
    eng.runner.ws.check()
    # sampled speculation runs too (temperature only)
    o2 = eng.generate(prompts[:1], SamplingParams(max_tokens=16, temperature=0.8, ignore_eos=True))[0]
    assert len(o2) == 16


def test_medusa_heads_int4_projection_matches_fp32(cuda):
    """On the GPU the heads' vocabulary projections are INT4 weights run by the W4A16 GEMM:
    logits against the fp32 heads with the dequantized projection."""
    from squish_b200._ext import native
    from squish_b200.engine.medusa import MedusaHeads

    cpu = MedusaHeads.random(256, 1000, num_heads=2, num_layers=1, seed=4)
    dev = MedusaHeads.from_state_dict(cpu.state_dict(), device=cuda)
    assert dev.quantized
    h = torch.randn(7, 256)
    got = dev.logits(h.to(cuda))
    for i, g in enumerate(got):
        sd = cpu.state_dict()
        u = sd[f"medusa_head.{i}.1.weight"]
        p, s, z = native().cpu.quantize_int4_asym(u, 64)
        uq = native().cpu.dequantize_int4_asym(p, s, z, 64)
        w, b = sd[f"medusa_head.{i}.0.linear.weight"], sd[f"medusa_head.{i}.0.linear.bias"]
        r = h.to(torch.bfloat16).float()
        r = r + torch.nn.functional.silu(r @ w.T + b)
        want = r @ uq.T
        err = (g.cpu() - want).abs().max().item()
        assert err <= 0.03 * want.abs().max().item(), err
