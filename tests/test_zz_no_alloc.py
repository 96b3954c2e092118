"""moe_align_static: the align entry point for callers that cannot allocate
device memory (a plugin handed only its input and output buffers, a server
whose memory pool is sealed after start-up). Its scratch is a static device
array inside the library, so the call itself allocates nothing.

Checked through the C ABI against the workspace-taking moe_align on two calls
in a row (the second must not see the first call's leftovers), plus the
size limit. Integer outputs, so the bar is bit-exact, as for moe_align.
"""
import numpy as np
import pytest
import torch

import mail_b200 as mb
from mail_b200 import _lib

pytestmark = pytest.mark.gpu


def routing_ids(seed, T, k, E):
    rng = np.random.default_rng(seed)
    ids = np.argsort(rng.random((T, E)), axis=1)[:, :k].astype(np.int32)
    ids[::7, 0] = -1  # dropped slots are part of the contract too
    return torch.from_numpy(ids).cuda()


def align_static(ids, E, block_m=128):
    """Calls moe_align_static with caller-owned outputs (no workspace)."""
    T, k = ids.shape
    S = T * k
    cap = int(_lib.query("moe_align_capacity", S, E, block_m))
    max_tiles = cap // block_m
    out = dict(
        sorted_slots=torch.full((max(cap, 1),), -7, dtype=torch.int32, device="cuda"),
        slot_pos=torch.full((max(S, 1),), -7, dtype=torch.int32, device="cuda"),
        group_sizes=torch.full((E,), -7, dtype=torch.int32, device="cuda"),
        padded_offsets=torch.full((E + 1,), -7, dtype=torch.int32, device="cuda"),
        tile_table=torch.full((int(_lib.query("moe_tile_table_ints", E, max_tiles)),), -7, dtype=torch.int32,
                              device="cuda"),
    )
    _lib.call("moe_align_static", ids.data_ptr(), T, k, E, block_m, out["sorted_slots"].data_ptr(),
              out["slot_pos"].data_ptr(), out["group_sizes"].data_ptr(), out["padded_offsets"].data_ptr(),
              out["tile_table"].data_ptr(), torch.cuda.current_stream().cuda_stream)
    out["slot_pos"] = out["slot_pos"][:S]
    return out


def assert_same_align(a, b, E):
    ta, tb = a["tile_table"].cpu().numpy(), b["tile_table"].cpu().numpy()
    n, rows = int(ta[0]), int(ta[1])
    assert tb[0] == n and tb[1] == rows and tb[2] == ta[2]
    np.testing.assert_array_equal(a["group_sizes"].cpu().numpy(), b["group_sizes"].cpu().numpy())
    np.testing.assert_array_equal(a["padded_offsets"].cpu().numpy(), b["padded_offsets"].cpu().numpy())
    np.testing.assert_array_equal(a["sorted_slots"][:rows].cpu().numpy(), b["sorted_slots"][:rows].cpu().numpy())
    np.testing.assert_array_equal(a["slot_pos"].cpu().numpy(), b["slot_pos"].cpu().numpy())
    mt = (len(ta) - 5 - E) // 2
    np.testing.assert_array_equal(ta[4:5 + E + n], tb[4:5 + E + n])
    np.testing.assert_array_equal(ta[5 + E + mt:5 + E + mt + n], tb[5 + E + mt:5 + E + mt + n])


def test_align_static_matches_align_on_two_calls_in_a_row():
    # first a larger problem, then a smaller one with more experts, so stale
    # histogram entries from the first call would corrupt the second
    for seed, (T, k, E) in enumerate([(8192, 8, 256), (300, 4, 300)]):
        ids = routing_ids(seed, T, k, E)
        got = align_static(ids, E)
        ref = mb.moe_align(ids, E, 128)
        torch.cuda.synchronize()
        assert_same_align(ref, got, E)
    assert mb.device_error() == 0


@pytest.mark.parametrize("T,k,E", [
    (16288, 8, 256),   # scratch 1,047,808 B: the last tail region ends just below the 1 MiB array
    (990, 8, 4096),    # more than 1024 experts: the multi-kernel path, scratch just under 1 MiB
    (60, 8, 4096),     # the same with fewer slots than experts
    (2048, 8, 128),    # 16384 slots: the one-CTA align, no scratch
])
def test_align_static_edges_match_align(T, k, E):
    lib = _lib.load()
    assert lib.moe_align_workspace_size(T, k, E, 128) <= (1 << 20)
    ids = routing_ids(T + E, T, k, E)
    for _ in range(2):
        got = align_static(ids, E)
        ref = mb.moe_align(ids, E, 128)
        torch.cuda.synchronize()
        assert_same_align(ref, got, E)
    assert mb.device_error() == 0


def test_align_static_rejects_requests_beyond_its_scratch():
    lib = _lib.load()
    T, k, E = 1 << 20, 8, 256  # 8M slots: far more scratch than the static array
    assert lib.moe_align_workspace_size(T, k, E, 128) > (1 << 20)
    fake = 256  # never dereferenced: the size check rejects the call first
    rc = lib.moe_align_static(fake, T, k, E, 128, fake, fake, fake, fake, fake, None)
    assert rc == 1
    assert "scratch" in lib.moe_last_error().decode()
