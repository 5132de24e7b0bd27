"""Tensor parallelism on 2 GPUs (skipped with fewer): the fused GEMM+all-reduce over NVLink
peer memory, the sequence-parallel GEMM->reduce-scatter / RMSNorm+all-gather / gather-waiting
GEMM, the expert-parallel all-to-all and the vocab gather against fp32 references, and the
tensor-parallel engine (fused, sequence-parallel and NCCL modes; dense and MoE) against the
CPU fp32 oracle."""
import dataclasses
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _collectives_worker(rank, world, port, q):
    _init(rank, world, port)
    try:
        from squish_b200 import ops
        from squish_b200._ext import native
        from squish_b200.parallel.comm import TPComm

        dev = torch.device("cuda", rank)
        H, V, Tmax = 1024, 4000, 256
        comm = TPComm("nvlink", Tmax, H, 64, V, device=dev)
        ws = ops.Workspace(dev)
        errs = []
        for T, K in ((1, 512), (7, 1024), (64, 768), (200, 512)):
            g = torch.Generator().manual_seed(T)  # same full weight on every rank
            wfull = torch.randn(H, K * world, generator=g) * 0.02
            x_full = torch.randn(T, K * world, generator=g)
            h0 = torch.randn(T, H, generator=g) * 0.1
            wl = wfull[:, rank * K:(rank + 1) * K].contiguous()
            p, s, z = native().cpu.quantize_int4_asym(wl, 64)
            w = ops.prepare_int4_weight(p, s, z, K, 64, dev)
            deq = native().cpu.dequantize_int4_asym(p, s, z, 64)
            x = x_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16)
            h = h0.to(torch.bfloat16).to(dev)
            for _ in range(3):  # repeated ops exercise the parity / flag reuse protocol
                hh = h.clone()
                comm.gemm_allreduce(x.to(dev), w, hh, ws)
            torch.cuda.synchronize()
            comm.check()
            # fp32 reference of this rank's partial, summed over ranks with an fp32 all_reduce
            part = (x.float() @ deq.T).to(dev)
            dist.all_reduce(part)
            want = h0.to(torch.bfloat16).float() + part.cpu()
            errs.append(float((hh.float().cpu() - want).abs().max()) / float(part.abs().max().cpu()))
            # every rank holds the same bits
            ref = hh.clone()
            dist.broadcast(ref, 0)
            assert torch.equal(ref, hh)
        # generic push all-reduce (expert-parallel partial outputs)
        for T in (3, 130):
            part = (torch.randn(T, H, generator=torch.Generator().manual_seed(rank * 100 + T)) * 0.1)
            base = torch.randn(T, H, generator=torch.Generator().manual_seed(T))
            hh = base.to(torch.bfloat16).to(dev)
            comm.allreduce_add(part.to(torch.bfloat16).to(dev), hh)
            torch.cuda.synchronize()
            tot = part.to(torch.bfloat16).float().to(dev)
            dist.all_reduce(tot)
            want = base.to(torch.bfloat16).float() + tot.cpu()
            # bf16 output: compare against the magnitude of the result, not of the partials
            errs.append(float((hh.float().cpu() - want).abs().max()) / float(want.abs().max()))
        comm.check()
        # vocab gather
        from squish_b200.parallel.shard import vocab_shard

        v0, v1 = vocab_shard(V, rank, world)
        full = torch.randn(5, V, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
        got = comm.gather_logits(full[:, v0:v1].contiguous().to(dev), 5)
        torch.cuda.synchronize()
        gather_ok = torch.equal(got.cpu(), full)
        comm.close()
        q.put((rank, errs, gather_ok))
    finally:
        dist.destroy_process_group()


def _sp_worker(rank, world, port, q):
    """Sequence-parallel collectives: GEMM -> reduce-scatter, the fused residual add + RMSNorm +
    all-gather, and the all-gather-waiting GEMM, against fp32 references (several row counts,
    including fewer rows than ranks and the bf16 large-M path)."""
    _init(rank, world, port)
    try:
        from squish_b200 import ops
        from squish_b200._ext import native
        from squish_b200.parallel.comm import TPComm

        dev = torch.device("cuda", rank)
        H, V, Tmax, K, F = 1024, 4000, 512, 512, 768
        comm = TPComm("sp", Tmax, H, 64, V, device=dev)
        ws = ops.Workspace(dev)
        errs = []
        for T in (1, 7, 64, 200, 448):
            g = torch.Generator().manual_seed(T)  # the same full tensors on every rank
            w_o = torch.randn(H, K * world, generator=g) * 0.02
            w_up = torch.randn(F, H, generator=g) * 0.02
            x_full = torch.randn(T, K * world, generator=g)
            h0 = torch.randn(T, H, generator=g)
            lnw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
            wl = w_o[:, rank * K:(rank + 1) * K].contiguous()
            p, s, z = native().cpu.quantize_int4_asym(wl, 64)
            wo = ops.prepare_int4_weight(p, s, z, K, 64, dev)
            deq = native().cpu.dequantize_int4_asym(p, s, z, 64)
            p2, s2, z2 = native().cpu.quantize_int4_asym(w_up, 64)
            wup = ops.prepare_int4_weight(p2, s2, z2, H, 64, dev)
            deq_up = native().cpu.dequantize_int4_asym(p2, s2, z2, 64)
            x = x_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16).to(dev)
            h = h0.to(torch.bfloat16).to(dev)
            for _ in range(3):  # repeated rounds exercise the parity / counter protocol
                hh = h.clone()
                e = comm.gemm_rs(x, wo, ws)
                comm.rs_norm_ag(hh, lnw.to(dev), 1e-6, T, e)
                y = comm.gemm_ag(wup, torch.empty(T, F, dtype=torch.bfloat16, device=dev), T, False, ws)
            torch.cuda.synchronize()
            comm.check()
            part = (x.float().cpu() @ deq.T).to(dev)
            dist.all_reduce(part)
            hsum = (h0.to(torch.bfloat16).float() + part.cpu()).to(torch.bfloat16).float()
            xn = (hsum * torch.rsqrt(hsum.pow(2).mean(-1, keepdim=True) + 1e-6) * lnw.float()).to(torch.bfloat16)
            R = -(-T // world)
            r0, r1 = rank * R, min(T, (rank + 1) * R)
            if r1 > r0:  # owned residual rows were updated
                errs.append(float((hh[r0:r1].float().cpu() - hsum[r0:r1]).abs().max()) / float(hsum.abs().max()))
            errs.append(float((comm.xg[:T].float().cpu() - xn.float()).abs().max()) / float(xn.float().abs().max()))
            want = xn.float() @ deq_up.T
            errs.append(float((y.float().cpu() - want).abs().max()) / float(want.abs().max()))
        comm.close()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def _ep_worker(rank, world, port, q):
    """Expert-parallel all-to-all (dispatch of the owned rows to the experts' ranks, local
    grouped INT4 experts, combine back through the reduce-scatter blocks, residual + RMSNorm)
    against an fp32 reference of the same experts with the GPU's own routing decisions."""
    _init(rank, world, port)
    try:
        from squish_b200 import ops
        from squish_b200.models.config import get_preset
        from squish_b200.models.moe import MoELayer, MoEScratch
        from squish_b200.models.weights import random_checkpoint
        from squish_b200.parallel.comm import TPComm
        from squish_b200.parallel.shard import shard_checkpoint

        dev = torch.device("cuda", rank)
        cfg, qc = get_preset("tiny-moe")
        ck = random_checkpoint(cfg, qc, seed=3, device="cpu")
        local = shard_checkpoint(ck, rank, world)
        lc = local.config
        H, Tmax, kk = cfg.hidden_size, 512, cfg.num_experts_per_tok
        comm = TPComm("sp", Tmax, H, 64, cfg.vocab_size, device=dev)
        comm.setup_ep(kk, lc.num_local_experts)
        layer = MoELayer.from_checkpoint(local, 0, dev, MoEScratch(lc, world * comm.sp_rows_max, dev))
        ws = ops.Workspace(dev)
        pre = "model.layers.0.mlp.experts."
        experts = {}

        def expert(e):
            if e not in experts:
                experts[e] = [ck[f"{pre}{e}.{n}.weight"].dequantize() for n in ("gate_proj", "up_proj", "down_proj")]
            return experts[e]

        wg = ck["model.layers.0.mlp.gate.weight"].data.to(torch.bfloat16).float()
        errs, route_ok = [], True
        for T in (1, 3, 64, 300):
            g = torch.Generator().manual_seed(T)  # the same rows on every rank
            x = torch.randn(T, H, generator=g).to(torch.bfloat16)
            h0 = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
            lnw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
            r0, own = comm.ep_own(T)
            h = h0.to(dev)
            for _ in range(3):  # repeated rounds exercise the counters and the buffer reuse
                hh = h.clone()
                comm.xg[r0:r0 + own].copy_(x[r0:r0 + own].to(dev))
                e = layer.forward_a2a(comm, comm.xg[r0:r0 + own], T, ws)
                comm.rs_norm_ag(hh, lnw.to(dev), 1e-6, T, e)
                comm.ag_wait(T)
            torch.cuda.synchronize()
            comm.check()
            if own == 0:
                continue
            ti = layer.scratch.ids[: own * kk].view(own, kk).cpu()
            tv = layer.scratch.w[: own * kk].view(own, kk).cpu()
            xf = x[r0:r0 + own].float()
            p = torch.softmax((xf @ wg.T).to(torch.bfloat16).float(), -1)
            route_ok &= bool((torch.gather(p, 1, ti.long()) >= p.topk(kk, -1).values[:, -1:] - 2e-2).all())
            out = h0[r0:r0 + own].float().clone()
            for t in range(own):
                for j in range(kk):
                    gw, uw, dw = expert(int(ti[t, j]))
                    a = (torch.nn.functional.silu(xf[t] @ gw.T) * (xf[t] @ uw.T)).to(torch.bfloat16).float()
                    out[t] += tv[t, j] * (a @ dw.T)
            got = hh[r0:r0 + own].float().cpu()
            scale = (out - h0[r0:r0 + own].float()).abs().max().item()
            errs.append(((got - out).abs().max().item() - 2e-3) / max(scale, 1e-6))
            # the owned rows of the gathered buffer hold RMSNorm of the stored residual rows
            xn = (got * torch.rsqrt(got.pow(2).mean(-1, keepdim=True) + 1e-6) * lnw.float()).to(torch.bfloat16)
            errs.append(float((comm.xg[r0:r0 + own].float().cpu() - xn.float()).abs().max())
                        / float(xn.float().abs().max()))
        comm.close()
        q.put((rank, errs, route_ok))
    finally:
        dist.destroy_process_group()


def _engine_worker(rank, world, port, mode, preset, q):
    _init(rank, world, port)
    try:
        from squish_b200.engine.engine import EngineConfig, LLMEngine
        from squish_b200.engine.sampling import SamplingParams
        from squish_b200.models.config import get_preset
        from squish_b200.models.weights import random_checkpoint

        cfg, qc = _preset(preset)
        ck = random_checkpoint(cfg, qc, seed=0)
        eng = LLMEngine.from_checkpoint(ck, torch.device("cuda", rank), EngineConfig(
            max_num_seqs=4, max_num_batched_tokens=128, max_model_len=256, num_pages=64, tp=world, tp_mode=mode))
        rng = np.random.default_rng(7)
        prompts = [rng.integers(0, cfg.vocab_size, 23).tolist(), rng.integers(0, cfg.vocab_size, 150).tolist()]
        outs = eng.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True))
        eng.comm.check()
        eng.graphs = None  # release graphs holding collectives before the group goes away
        eng.comm.close()
        q.put((rank, prompts, outs))
    finally:
        dist.destroy_process_group()


def _run(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(world)], key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def _preset(name):
    from squish_b200.models.config import get_preset

    cfg, qc = get_preset(name)
    if name == "tiny-moe":
        return dataclasses.replace(cfg, tie_embeddings=False), qc
    return dataclasses.replace(cfg, tie_embeddings=False, intermediate_size=512), qc


needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


@needs2
def test_fused_gemm_allreduce_and_gather():
    res = _run(_collectives_worker, 2)
    for rank, errs, gather_ok in res:
        assert gather_ok
        assert max(errs) < 2e-2, errs


@needs2
def test_sequence_parallel_collectives():
    res = _run(_sp_worker, 2)
    for rank, errs in res:
        assert max(errs) < 2e-2, errs


@needs2
def test_expert_parallel_all_to_all():
    res = _run(_ep_worker, 2)
    for rank, errs, route_ok in res:
        assert route_ok
        assert max(errs) < 2e-2, errs


@needs2
@pytest.mark.parametrize("mode,preset", [("nvlink", "tiny-llama"), ("nccl", "tiny-llama"), ("sp", "tiny-llama"),
                                         ("nvlink", "tiny-moe"), ("nccl", "tiny-moe"), ("sp", "tiny-moe")])
def test_tp_engine_matches_oracle(mode, preset):
    from squish_b200.models.reference import ReferenceModel
    from squish_b200.models.weights import random_checkpoint

    from .test_engine_gpu import _teacher_forced_ok

    res = _run(_engine_worker, 2, mode, preset)
    assert res[0][2] == res[1][2]
    cfg, qc = _preset(preset)
    ref = ReferenceModel(random_checkpoint(cfg, qc, seed=0))
    for p, o in zip(res[0][1], res[0][2]):
        ok, worst = _teacher_forced_ok(ref, p, o)
        assert ok, (worst, o)
