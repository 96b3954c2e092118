"""The one-launch decode kernel (MOE_OPT_DECODE_FUSED): at most 16 tokens and
128 routed slots run as one persistent kernel — routing, gate_up GEMM +
SwiGLU, down GEMM + weighted combine and the output conversion as phases
whose CTAs hand results on through counters (a launch counter in the
library's memory, counts in the workspace). Checked against the oracle (max-abs-rel
error 1e-2, the bar of every bf16 output here) and against the multi-launch
path on the same inputs."""
import numpy as np
import pytest
import torch

import mail_b200 as mb
from mail_b200 import _lib
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-2


def dev():
    return torch.device("cuda", 0)


def max_abs_rel(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def layer(T, H, I, E, dtype, seed):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((T, H), dtype=np.float32)).to(dev(), dtype)
    w13 = torch.from_numpy(rng.standard_normal((E, 2 * I, H), dtype=np.float32) * 0.02).to(dev(), dtype)
    w2 = torch.from_numpy(rng.standard_normal((E, H, I), dtype=np.float32) * 0.02).to(dev(), dtype)
    return x, w13.transpose(1, 2), w2.transpose(1, 2)


def run(x, w13, w2, ids, wts, fused=True):
    lib = _lib.load()
    old = lib.moe_get_option(_lib.OPT_DECODE_FUSED)
    assert lib.moe_set_option(_lib.OPT_DECODE_FUSED, int(fused)) == 0
    try:
        before = lib.moe_launch_count()
        y = mb.fused_moe_mlp(x, w13, w2, torch.from_numpy(wts).to(dev()), torch.from_numpy(ids).to(dev()))
        launches = lib.moe_launch_count() - before
    finally:
        lib.moe_set_option(_lib.OPT_DECODE_FUSED, old)
    return y, launches


def oracle(x, w13, w2, ids, wts, dtype):
    rnd = O.round_bf16 if dtype == torch.bfloat16 else O.round_fp16
    return O.moe_mlp_topk(x.float().cpu().numpy(), w13.float().cpu().numpy(), w2.float().cpu().numpy(), wts, ids,
                          round_hidden=rnd)


@pytest.mark.parametrize("T,H,I,E,k,routing,dtype", [
    (1, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16),     # one token: gate_up K split 3 ways
    (3, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16),
    (8, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16),
    (16, 2048, 768, 128, 8, "zipf1.2", torch.bfloat16),    # 128 slots: the largest one-launch batch
    (16, 1024, 512, 8, 2, "uniform-softmax", torch.bfloat16),  # many tokens per expert
    (5, 512, 136, 16, 4, "sigmoid", torch.float16),        # ragged I (a partial feature tile), fp16
    (2, 4096, 1536, 64, 6, "hot25-zipf1.0", torch.bfloat16),
    (7, 1032, 264, 257, 8, "uniform-softmax", torch.bfloat16),  # H, I not multiples of 64; odd E
])
def test_one_launch_matches_oracle_and_multi_launch(T, H, I, E, k, routing, dtype):
    x, w13, w2 = layer(T, H, I, E, dtype, T + H)
    ids, wts = O.synthetic_routing(routing, T, E, k, 3)
    y, launches = run(x, w13, w2, ids, wts, fused=True)
    assert launches == 1
    ref = oracle(x, w13, w2, ids, wts, dtype)
    assert max_abs_rel(y.float().cpu().numpy(), ref) < TOL
    y2, launches2 = run(x, w13, w2, ids, wts, fused=False)
    assert launches2 > 1
    assert max_abs_rel(y.float().cpu().numpy(), y2.float().cpu().numpy()) < TOL
    assert mb.device_error(dev()) == 0


def test_dropped_and_repeated_ids():
    """Ids outside [0, E) are dropped (a token with none left gets a zero
    row), and a token listing one expert twice gets both weights."""
    T, H, I, E, k = 12, 1024, 256, 32, 6
    x, w13, w2 = layer(T, H, I, E, torch.bfloat16, 5)
    ids, wts = O.synthetic_routing("uniform-softmax", T, E, k, 6)
    ids = ids.copy()
    ids[[0, 9]] = -1                  # every slot dropped
    ids[3, :3] = E + 2                # some dropped
    ids[5, 1] = ids[5, 0]             # one expert twice
    y, launches = run(x, w13, w2, ids, wts)
    assert launches == 1
    yf = y.float().cpu().numpy()
    assert (yf[[0, 9]] == 0).all()
    assert max_abs_rel(yf, oracle(x, w13, w2, ids, wts, torch.bfloat16)) < TOL
    assert mb.device_error(dev()) == 0


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("distinct", [0, 1, 2, 3, 5, 8])
def test_one_token_few_experts(distinct, mode):
    """One token whose eight slots name only a few distinct experts (repeated
    ids; none valid for distinct = 0). Mode 1: the gate_up K splits of a
    feature tile run as one cluster and add their sums through the leader's
    shared memory; mode 2: no clusters, the split count follows the experts
    actually routed (up to 8 CTAs per feature tile), sums through global
    memory. Both add the splits in K order."""
    T, H, I, E, k = 1, 2048, 768, 128, 8
    x, w13, w2 = layer(T, H, I, E, torch.bfloat16, 40 + distinct)
    rng = np.random.default_rng(distinct)
    experts = rng.choice(E, size=max(distinct, 1), replace=False)
    ids = np.array([[experts[j % len(experts)] for j in range(k)]], dtype=np.int32)
    if distinct == 0:
        ids[:] = -1
    wts = rng.random((1, k)).astype(np.float32)
    wts /= wts.sum()
    y, launches = run(x, w13, w2, ids, wts, fused=mode)
    assert launches == 1
    yf = y.float().cpu().numpy()
    if distinct == 0:
        assert (yf == 0).all()
    else:
        assert max_abs_rel(yf, oracle(x, w13, w2, ids, wts, torch.bfloat16)) < TOL
    assert mb.device_error(dev()) == 0


def test_launch_counter_over_many_launches_of_different_grids():
    """Consecutive launches with different grid sizes (the launch counter
    counts the CTAs of each launch and tags its counts) stay correct and
    raise no device error."""
    H, I, E = 2048, 768, 128
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    outs = []
    for rep in range(30):
        T = (1, 2, 16, 5, 9)[rep % 5]
        x = torch.randn(T, H, device=dev()).to(torch.bfloat16)
        ids, wts = O.synthetic_routing("zipf1.2", T, E, 8, rep)
        y, _ = run(x, w13, w2, ids, wts)
        outs.append((x, ids, wts, y))
    torch.cuda.synchronize()
    assert mb.device_error(dev()) == 0
    for x, ids, wts, y in outs[-5:]:
        assert max_abs_rel(y.float().cpu().numpy(), oracle(x, w13, w2, ids, wts, torch.bfloat16)) < TOL


def test_graph_replay_of_the_one_launch_path():
    T, H, I, E, k = 4, 2048, 768, 128, 8
    w13 = (torch.randn(E, 2 * I, H, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    w2 = (torch.randn(E, H, I, device=dev()) * 0.02).to(torch.bfloat16).transpose(1, 2)
    cap = mb.CapturedMoeMLP(w13, w2, T, k, dtype=torch.bfloat16)
    assert cap.kernels == 1
    for seed in range(3):
        x = torch.randn(T, H, device=dev()).to(torch.bfloat16)
        ids, wts = O.synthetic_routing("zipf1.2", T, E, k, 20 + seed)
        ids_t, wts_t = torch.from_numpy(ids).to(dev()), torch.from_numpy(wts).to(dev())
        got = cap(x, wts_t, ids_t).float()
        ref = mb.fused_moe_mlp(x, w13, w2, wts_t, ids_t).float()
        assert max_abs_rel(got.cpu().numpy(), ref.cpu().numpy()) < TOL
    assert mb.device_error(dev()) == 0
