"""Expert parallelism over peer memory, emulated for W ranks on one GPU.

Every rank's buffers live on the same device and the "peer" pointer tables
point at them, so the dispatch kernel's and the down GEMM's cross-rank stores
exercise exactly the index path of the multi-GPU run (no kernel waits on
another: the ranks' launches are serialised on one stream). Checked against
the single-GPU fused op on all experts (same tolerance as the other bf16
tests) and, for the plan, bit-exactly against the oracle's layout.
"""
import ctypes

import numpy as np
import pytest
import torch

import mail_b200 as mb
from mail_b200 import _lib
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = torch.device("cuda", 0)


def st():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("W,E,seed", [(2, 8, 0), (4, 8, 1), (8, 64, 2), (3, 9, 3)])
def test_ep_plan_matches_oracle(W, E, seed):
    rng = np.random.default_rng(seed)
    counts = rng.integers(0, 400, size=(W, E)).astype(np.int32)
    counts[:, 1] = 0  # an expert nobody routes to
    EL = E // W
    recv_cap = int(_lib.query("moe_align_capacity", int(counts.sum()) , EL, 128)) + 128 * E
    max_tiles = recv_cap // 128
    c_dev = torch.from_numpy(counts).to(DEV)
    for r in range(W):
        ref = O.ep_plan(counts, r, EL)
        dest = torch.empty(E, dtype=torch.int32, device=DEV)
        table = torch.empty(int(_lib.query("moe_tile_table_ints", EL, max_tiles)), dtype=torch.int32, device=DEV)
        meta = torch.zeros(recv_cap, dtype=torch.int32, device=DEV)
        _lib.call("moe_ep_plan", c_dev.data_ptr(), W, r, E, None, 0, dest.data_ptr(), table.data_ptr(), max_tiles,
                  meta.data_ptr(), recv_cap, None, st())
        t = table.cpu().numpy()
        n = len(ref["tile_row_start"])
        np.testing.assert_array_equal(dest.cpu().numpy(), ref["dest_base"])
        assert t[0] == n and t[1] == ref["total_rows"] and t[2] == 0
        np.testing.assert_array_equal(t[4:5 + EL], ref["tile_cumsum"])
        np.testing.assert_array_equal(t[5 + EL:5 + EL + n], ref["tile_row_start"])
        np.testing.assert_array_equal(t[5 + EL + max_tiles:5 + EL + max_tiles + n], ref["tile_row_count"])
        m = meta.cpu().numpy()
        for s0, c0 in zip(ref["tile_row_start"], ref["tile_row_count"]):
            assert (m[s0 + c0:s0 + 128] == -1).all()


def _ptrs(ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=DEV)


@pytest.mark.parametrize("W,E,k,T,quant,rep", [(2, 8, 2, 300, False, ()), (4, 8, 2, 256, False, ()),
                                                (2, 16, 4, 200, True, ()), (4, 8, 2, 256, False, (6, 1)),
                                                (2, 16, 4, 200, True, (3,))])
def test_ep_emulated_ranks_match_single_gpu(W, E, k, T, quant, rep):
    """rep: experts replicated on every rank (mail_b200.ep.ExpertPlacement):
    the exchange then runs over virtual expert ids, owned experts first, then
    the replicas, and a replicated expert's slots stay on their own rank."""
    from mail_b200.ep import ExpertPlacement
    H, I = 512, 256
    E_glob = E
    places = [ExpertPlacement(E, W, r, rep) for r in range(W)]
    EL_own = E // W
    EL = places[0].EL_virtual
    E = places[0].E_virtual
    g = torch.Generator(device=DEV).manual_seed(11)
    w13 = (torch.randn(E_glob, 2 * I, H, device=DEV, generator=g) * 0.03).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E_glob, H, I, device=DEV, generator=g) * 0.03).to(torch.bfloat16).transpose(1, 2)
    scales = None
    if quant:
        w13, w2, scales = mb.quantize_weights_int8(w13, w2)
    xs, idss, wtss = [], [], []
    for r in range(W):
        rng = np.random.default_rng(100 + r)
        xs.append(torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(DEV, torch.bfloat16))
        ids, wts = O.synthetic_routing("uniform-softmax", T, E_glob, k, seed=r)
        ids[::6, 0] = -1
        if rep:
            ids[1::3, 1] = rep[0]  # make the first replicated expert hot
        idss.append(torch.from_numpy(ids).to(DEV))
        wtss.append(torch.from_numpy(wts).to(DEV))
    S = T * k
    recv_cap = int(_lib.query("moe_align_capacity", W * S, EL, 128))
    max_tiles = recv_cap // 128
    recv_code = _lib.I8 if quant else _lib.BF16
    recv_x = [torch.empty((recv_cap, H), dtype=torch.int8 if quant else torch.bfloat16, device=DEV) for _ in range(W)]
    recv_s = [torch.empty(recv_cap, dtype=torch.float32, device=DEV) for _ in range(W)]
    meta = [torch.full((recv_cap,), -5, dtype=torch.int32, device=DEV) for _ in range(W)]
    ret = [torch.empty((S, H), dtype=torch.bfloat16, device=DEV) for _ in range(W)]
    vids = [places[r].remap(idss[r]).contiguous() for r in range(W)]
    aligns = [mb.moe_align(vids[r], E, 1) for r in range(W)]
    counts = torch.stack([a["group_sizes"] for a in aligns])
    tables, dests, rets = [], [], []
    for r in range(W):
        dest = torch.empty(E, dtype=torch.int32, device=DEV)
        table = torch.empty(int(_lib.query("moe_tile_table_ints", EL, max_tiles)), dtype=torch.int32, device=DEV)
        rp = torch.empty(S, dtype=torch.int32, device=DEV)
        _lib.call("moe_ep_plan", counts.data_ptr(), W, r, E, aligns[r]["slot_pos"].data_ptr(), S, dest.data_ptr(),
                  table.data_ptr(), max_tiles, meta[r].data_ptr(), recv_cap, rp.data_ptr(), st())
        tables.append(table), dests.append(dest), rets.append(rp)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    px, ps, pm, pr = _ptrs(recv_x), _ptrs(recv_s), _ptrs(meta), _ptrs(ret)
    for r in range(W):
        a = aligns[r]
        _lib.call("moe_ep_dispatch", xs[r].data_ptr(), _lib.BF16, H, k, vids[r].data_ptr(), a["sorted_slots"].data_ptr(),
                  a["padded_offsets"].data_ptr(), dests[r].data_ptr(), a["tile_table"][1:2].data_ptr(), S, W, r, EL,
                  recv_cap, px.data_ptr(), recv_code, ps.data_ptr() if quant else None, pm.data_ptr(), err.data_ptr(),
                  st())
    w13k, w2k = mb.kmajor(w13), mb.kmajor(w2)
    ws = torch.empty(_lib.query("moe_ep_expert_pass_workspace_size", recv_cap, I, recv_code), dtype=torch.uint8,
                     device=DEV)
    for r in range(W):
        # this rank's owned experts, then its replica copies
        own = list(range(r * EL_own, (r + 1) * EL_own)) + list(rep)
        w13r, w2r = w13k[own].contiguous(), w2k[own].contiguous()
        s13 = scales[0][own].contiguous() if quant else None
        s2 = scales[1][own].contiguous() if quant else None
        _lib.call("moe_ep_expert_pass", recv_x[r].data_ptr(), recv_code, recv_s[r].data_ptr() if quant else None,
                  recv_cap, H, w13r.data_ptr(), w2r.data_ptr(), EL, I,
                  s13.data_ptr() if quant else None, s2.data_ptr() if quant else None, tables[r].data_ptr(),
                  meta[r].data_ptr(), pr.data_ptr(), W, S, _lib.BF16, ws.data_ptr(), ws.numel(), st())
    assert int(err.item()) == 0
    for r in range(W):
        y = torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
        _lib.call("moe_combine_rows", ret[r].data_ptr(), _lib.BF16, H, rets[r].data_ptr(), wtss[r].data_ptr(), T, k,
                  y.data_ptr(), _lib.BF16, st())
        y_ref = mb.fused_moe_mlp(xs[r], w13, w2, wtss[r], idss[r], scales=scales)
        err_r = float((y.float() - y_ref.float()).abs().max() / y_ref.float().abs().max())
        assert err_r < TOL, (r, err_r)
    assert mb.device_error(DEV) == 0
