"""bench.py builds its synthetic routing itself (the GPU arm does not use the
oracle); the CPU-baseline leg uses the oracle's generator. Both must produce
the same workload."""
import numpy as np
import pytest

import bench
from oracle import moe_oracle as O


@pytest.mark.parametrize("name,T,E,k", [("uniform-softmax", 300, 8, 2), ("sigmoid", 77, 256, 8),
                                        ("zipf1.2", 33, 128, 8), ("hot25-zipf1.0", 200, 64, 6)])
@pytest.mark.parametrize("seed", [0, 1, 7919 * 3])
def test_bench_routing_equals_oracle(name, T, E, k, seed):
    ids, w = bench.make_routing(name, T, E, k, seed)
    ids_o, w_o = O.synthetic_routing(name, T, E, k, seed)
    np.testing.assert_array_equal(ids, ids_o)
    np.testing.assert_array_equal(w, w_o)
    assert ids.dtype == np.int32 and w.dtype == np.float32
