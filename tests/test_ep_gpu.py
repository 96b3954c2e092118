"""Expert-parallel layer on 2 GPUs (NCCL): matches the single-GPU fused op on
the same weights and tokens, also with replicated experts. Skipped when fewer
than 2 GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg, transport, q):
    import torch.distributed as dist
    from datetime import timedelta

    import mail_b200 as mb
    from mail_b200.ep import ExpertParallelMoE
    from oracle import moe_oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        T, H, I, E, k, quant, repl = cfg
        g = torch.Generator(device=dev).manual_seed(7)  # identical global weights on every rank
        w13 = (torch.randn(E, 2 * I, H, device=dev, generator=g) * 0.02).to(torch.bfloat16).transpose(1, 2)
        w2 = (torch.randn(E, H, I, device=dev, generator=g) * 0.02).to(torch.bfloat16).transpose(1, 2)
        scales = None
        if quant:
            w13, w2, scales = mb.quantize_weights_int8(w13, w2)
        rng = np.random.default_rng(rank)
        x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev, torch.bfloat16)
        ids, wts = O.synthetic_routing("uniform-softmax", T, E, k, seed=rank)
        ids[::5, 0] = -1
        ids_t, wts_t = torch.from_numpy(ids).to(dev), torch.from_numpy(wts).to(dev)
        el = E // world
        lsc = None if scales is None else tuple(s[rank * el:(rank + 1) * el] for s in scales)
        rl = list(repl)
        replicas = None
        if rl:  # every rank also holds these experts and serves its own slots to them
            replicas = (rl, w13[rl], w2[rl], None if scales is None else tuple(s[rl] for s in scales))
        if transport == "peer":
            from mail_b200.ep import PeerExpertParallelMoE
            layer = PeerExpertParallelMoE(w13[rank * el:(rank + 1) * el], w2[rank * el:(rank + 1) * el], E,
                                          max_tokens=T, top_k=k, scales=lsc, replicas=replicas)
        else:
            layer = ExpertParallelMoE(w13[rank * el:(rank + 1) * el], w2[rank * el:(rank + 1) * el], E,
                                      scales=lsc, chunks=2, min_chunk_tokens=128, replicas=replicas)
        y = layer(x, wts_t, ids_t)
        y_again = layer(x, wts_t, ids_t)  # the second call reuses the buffers
        torch.cuda.synchronize()
        assert torch.equal(y, y_again)
        if transport == "peer":
            assert not layer.overflowed()
            layer.close()
        y_ref = mb.fused_moe_mlp(x, w13, w2, wts_t, ids_t, scales=scales)
        torch.cuda.synchronize()
        err = float((y.float() - y_ref.float()).abs().max() / y_ref.float().abs().max())
        q.put((rank, err, mb.device_error(dev)))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["peer", "nccl"])
@pytest.mark.parametrize("cfg", [(512, 1024, 512, 8, 2, False, ()), (300, 1024, 256, 16, 4, True, ()),
                                 (512, 1024, 512, 8, 2, False, (5,)), (300, 1024, 256, 16, 4, True, (0, 9))])
def test_expert_parallel_matches_single_gpu(cfg, transport):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, cfg, transport, q)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=240)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    for _ in range(world):
        rank, err, derr = q.get(timeout=5)
        assert derr == 0
        assert err < TOL, (rank, err)
