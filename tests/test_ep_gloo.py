"""Expert-parallel exchange logic as world_size-2 gloo ranks on CPU.

The device kernels are replaced by oracle-backed stand-ins (test
infrastructure); the dispatch plan, count exchange, all-to-all routing of
rows, return path and combine indexing are the product's own code
(mail_b200.ep) and must reproduce the single-process oracle exactly up to
fp32 summation order.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as O


class OracleOps:
    """CPU stand-ins for the CUDA ops of mail_b200.ep.CudaOps."""

    def sort_slots(self, topk_ids, num_experts):
        a = O.align(topk_ids.numpy(), num_experts, 1)
        n_valid = torch.tensor([int(a["padded_offsets"][-1])], dtype=torch.int32)
        return (torch.from_numpy(a["sorted_slots"]), torch.from_numpy(a["slot_pos"]),
                torch.from_numpy(a["group_sizes"]), n_valid)

    def gather(self, x, sorted_slots, top_k, rows, rows_dev=None):
        n = min(rows, int(rows_dev[0])) if rows_dev is not None else rows
        out = torch.zeros((rows, x.shape[1]), dtype=x.dtype)
        s = sorted_slots[:n].to(torch.int64)
        out[:n] = x[s // top_k]
        return out

    def expert_forward(self, x_rows, local_ids, w13, w2, scales):
        ids = local_ids.numpy().reshape(-1, 1)
        y = O.moe_mlp_topk(x_rows.numpy(), w13.numpy(), w2.numpy(), np.ones_like(ids, np.float32), ids)
        return torch.from_numpy(y)

    def combine(self, o_back, slot_pos, topk_weights, out_dtype, out=None):
        T, k = topk_weights.shape
        y = torch.zeros((T, o_back.shape[1]), dtype=torch.float32)
        pos = slot_pos.view(T, k).to(torch.int64)
        for j in range(k):
            m = pos[:, j] >= 0
            y[m] += topk_weights[m, j:j + 1] * o_back[pos[m, j]]
        if out is not None:
            out.copy_(y)
            return out
        return y.to(out_dtype)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, E, T, H, I, k, drop, chunks, result_q, replicated=()):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mail_b200.ep import ExpertParallelMoE
        rng = np.random.default_rng(100)  # same global weights on every rank
        w13 = rng.standard_normal((E, H, 2 * I), dtype=np.float32) * 0.1
        w2 = rng.standard_normal((E, I, H), dtype=np.float32) * 0.1
        rr = np.random.default_rng(rank)  # rank-local tokens and routing
        x = rr.standard_normal((T, H), dtype=np.float32)
        ids, wts = O.synthetic_routing("uniform-softmax", T, E, k, seed=rank)
        if drop:
            ids[::4, 0] = -1
        el = E // world
        rep = list(replicated)
        replicas = (rep, torch.from_numpy(w13[rep]), torch.from_numpy(w2[rep])) if rep else None
        layer = ExpertParallelMoE(torch.from_numpy(w13[rank * el:(rank + 1) * el]),
                                  torch.from_numpy(w2[rank * el:(rank + 1) * el]), E, ops=OracleOps(),
                                  chunks=chunks, min_chunk_tokens=8, replicas=replicas)
        y = layer(torch.from_numpy(x), torch.from_numpy(wts), torch.from_numpy(ids))
        ref = O.moe_mlp_topk(x, w13, w2, wts, ids)
        result_q.put((rank, float(np.abs(y.numpy() - ref).max()), float(np.abs(ref).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("E,T,k,drop,chunks,replicated", [(8, 40, 2, False, 1, ()), (4, 33, 3, True, 3, ()),
                                                           (6, 1, 2, False, 2, ()), (8, 64, 2, True, 2, ()),
                                                           (8, 40, 2, False, 1, (5,)), (4, 33, 3, True, 3, (0, 3)),
                                                           (8, 64, 2, True, 2, (6, 1, 2))])
def test_expert_parallel_two_ranks_matches_oracle(E, T, k, drop, chunks, replicated):
    """Replicated experts (one owned by each rank, in the last cases) run on
    the rank whose token routes to them; results stay those of the oracle."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, E, T, 32, 24, k, drop, chunks, q, replicated))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, err, scale in res:
        assert err <= 1e-5 * max(scale, 1.0), (rank, err, scale)
