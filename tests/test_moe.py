"""Mixture-of-experts MLP: routing, the engine's MoE decoder (lossless speculative decoding with EAGLE-3 and Medusa),
expert parallelism over Gloo ranks, and the CUDA routing / grouped-GEMM kernels against the PyTorch reference."""

import os

import pytest
import torch
import torch.multiprocessing as mp

import economize_b200 as eco
from economize_b200.models.config import tiny_llama
from economize_b200.models.llama import CausalLM, init_weights
from economize_b200.parallel.moe import ExpertParallel, moe_mlp, moe_reference, route, shard_experts
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.medusa import MedusaConfig

from .helpers import prompts, reference_greedy


def tiny_moe(seed: int = 0, device="cpu", dtype=torch.float32) -> CausalLM:
    cfg = tiny_llama(num_experts=4, experts_per_token=2, intermediate_size=128, model_type="mixtral")
    return init_weights(CausalLM(cfg, dtype, device), seed=seed)


def test_route_renormalises():
    logits = torch.tensor([[0.0, 3.0, 1.0, 2.0]])
    ids, w = route(logits, 2)
    assert ids.tolist() == [[1, 3]] and torch.allclose(w.sum(-1), torch.ones(1))


def test_moe_matches_dense_loop():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 16, generator=g)
    router = torch.randn(4, 16, generator=g)
    gu = torch.randn(4, 24, 16, generator=g) * 0.1
    down = torch.randn(4, 16, 12, generator=g) * 0.1
    out = moe_mlp(x, router, gu, down, 2)
    ids, w = route(x @ router.t(), 2)
    exp = torch.zeros(5, 16)
    for t in range(5):
        for j in range(2):
            e = int(ids[t, j])
            a, b = (x[t] @ gu[e].t()).chunk(2)
            exp[t] += w[t, j] * ((torch.nn.functional.silu(a) * b) @ down[e].t())
    torch.testing.assert_close(out, exp, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("config", [Eagle3Config(), MedusaConfig(num_heads=4)])
def test_moe_model_decodes_losslessly(config):
    model = tiny_moe()
    eff = eco.apply(model, config, decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((16,))[0]
    assert torch.equal(eff.decode(p, 10).tokens, reference_greedy(model, p, 10))


def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        x_all = torch.randn(2 * 6, 16, generator=g)
        router = torch.randn(4, 16, generator=g)
        gu = torch.randn(4, 24, 16, generator=g) * 0.1
        down = torch.randn(4, 16, 12, generator=g) * 0.1
        x = x_all[rank * 6:(rank + 1) * 6]
        ep = ExpertParallel(rank, world)
        own = ep.owned(4)
        out = moe_mlp(x, router, gu[own.start:own.stop], down[own.start:own.stop], 2, ep)
        exp = moe_reference(x, router, gu, down, 2)
        q.put((rank, float((out - exp).abs().max())))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.slow
def test_expert_parallel_matches_single_rank():
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(err < 1e-5 for _, err in res), res


def test_shard_experts_keeps_own_block():
    model = tiny_moe()
    full = model.layers[0].w_gate_up.detach().clone()
    shard_experts(model, ExpertParallel(1, 2))
    assert torch.equal(model.layers[0].w_gate_up, full[2:4])


# ---- GPU ------------------------------------------------------------------------------------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("T,E,k,H,F", [(1, 8, 2, 512, 1024), (61, 8, 2, 4096, 1024), (300, 16, 4, 1024, 512)])
def test_moe_kernels_match_reference(cuda, T, E, k, H, F):
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(T, H, device=cuda, generator=g).bfloat16()
    router = (torch.randn(E, H, device=cuda, generator=g) * 0.05).bfloat16()
    gu = (torch.randn(E, 2 * F, H, device=cuda, generator=g) * 0.02).bfloat16()
    down = (torch.randn(E, H, F, device=cuda, generator=g) * 0.02).bfloat16()
    out = moe_mlp(x, router, gu, down, k)
    from economize_b200 import ops

    logits = ops.linear(x, router).float()  # route like the kernel path (bf16 router logits)
    exp = moe_reference(x.float(), router.float(), gu.float(), down.float(), k, logits=logits)
    torch.testing.assert_close(out.float(), exp, atol=3e-2, rtol=3e-2)


@pytest.mark.gpu
def test_moe_route_positions_are_a_permutation(cuda):
    from economize_b200.ops._ext import require

    logits = torch.randn(200, 8, device=cuda).bfloat16()
    ids, w, pos, offsets = require().moe_route(logits, 2)
    assert sorted(pos.flatten().tolist()) == list(range(400))
    assert offsets[-1].item() == 400
    # the chosen experts carry the two largest logits (bf16 logits tie often; the kernel breaks ties by lower id)
    lf = logits.float()
    chosen = lf.gather(1, ids.long())
    top2 = lf.topk(2, -1).values
    assert torch.equal(chosen.sort(-1).values, top2.sort(-1).values)
    probs = torch.softmax(lf, -1).gather(1, ids.long())
    torch.testing.assert_close(w, probs / probs.sum(-1, keepdim=True), atol=1e-5, rtol=1e-4)


@pytest.mark.gpu
def test_moe_model_decodes_on_gpu(cuda):
    cfg = tiny_llama(num_experts=4, experts_per_token=2, hidden_size=512, head_dim=128, num_heads=4,
                     num_kv_heads=2, intermediate_size=512, model_type="mixtral")
    model = init_weights(CausalLM(cfg, torch.bfloat16, cuda), seed=0)
    eff = eco.apply(model, MedusaConfig(num_heads=4), decoding=eco.DecodeConfig(cycle_length=5, cuda_graphs=True))
    p = prompts((20,))[0].to(cuda)
    plain = eff.decode(p, 16, decoding=eco.DecodeConfig(cycle_length=1)).tokens
    assert torch.equal(eff.decode(p, 16).tokens.cpu(), plain.cpu())


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,k,H,F", [(1, 8, 2, 512, 1024), (61, 8, 2, 1024, 512), (40, 4, 4, 512, 256)])
def test_fused_ep_single_rank_matches_kernel_path(cuda, T, E, k, H, F):
    """The peer-store dispatch / segments / combine kernels with one rank (its own buffer as the only peer), over
    several calls (the arrival counters advance per call) and under CUDA-graph replay."""
    from economize_b200 import ops
    from economize_b200.ops._ext import require

    C = require()
    g = torch.Generator(device=cuda).manual_seed(T)
    router = (torch.randn(E, H, device=cuda, generator=g) * 0.05).bfloat16()
    gu = (torch.randn(E, 2 * F, H, device=cuda, generator=g) * 0.02).bfloat16()
    down = (torch.randn(E, H, F, device=cuda, generator=g) * 0.02).bfloat16()
    cap = 64 * k
    own, _ = C.symm_alloc(C.ep_buffer_bytes(1, E, cap, H, cap))

    def fused(x):
        _, w, pos, off = C.moe_route(ops.linear(x, router), k)
        return C.ep_moe(C.moe_gather(x, pos), off, pos, w, gu, down, [own], 0, cap, cap)

    try:
        for n in (T, max(T // 2, 1), T):
            x = torch.randn(n, H, device=cuda, generator=g).bfloat16()
            torch.testing.assert_close(fused(x).float(), moe_mlp(x, router, gu, down, k).float(), atol=2e-2, rtol=2e-2)
        static = torch.randn(T, H, device=cuda, generator=g).bfloat16()
        fused(static)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = fused(static)
        for _ in range(3):
            static.copy_(torch.randn(T, H, device=cuda, generator=g).bfloat16())
            graph.replay()
            torch.testing.assert_close(out.float(), moe_mlp(static, router, gu, down, k).float(), atol=2e-2,
                                       rtol=2e-2)
        torch.cuda.synchronize()
        assert C.status(cuda.index or 0) == 0
        del graph
    finally:
        torch.cuda.synchronize()
        C.symm_free(own)
