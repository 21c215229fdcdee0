"""PKM router on the GPU against the oracle: addresses and adapter ids must be
bit-exact (the benchmark requires results that match the CPU reference bit-exactly)."""
import numpy as np
import pytest

import oracle
import ti_b200 as ti

pytestmark = pytest.mark.gpu


def _oracle_assign(c1, c2, q):
    n, D = c1.shape
    addr = np.empty(len(q), np.int32)
    oracle.lib().orc_pkm_assign(oracle.ptr(c1), oracle.ptr(c2), n, D, oracle.ptr(q), len(q), oracle.ptr(addr))
    return addr


def _oracle_table(c1, c2, cents, ids):
    n = c1.shape[0]
    ca = _oracle_assign(c1, c2, cents)
    table = np.full(n * n, -1, np.int32)
    for a, i in zip(ca, ids):
        if table[a] < 0 or i < table[a]:
            table[a] = i
    return table


@pytest.mark.parametrize("n_queries", [8192, 65536])
def test_pkm_bench_shape_bit_exact(n_queries):
    # benchmark configuration 4: two 512 x 256 fp32 codebooks ~ N(0,1), 4096 adapter centroids
    c1 = oracle.fill_f32("pkm.c1", (512, 256), 0, 1.0)
    c2 = oracle.fill_f32("pkm.c2", (512, 256), 0, 1.0)
    cents = oracle.fill_f32("pkm.centroids", (4096, 512), 0, 1.0)
    q = oracle.fill_f32("pkm.queries", (n_queries, 512), 0, 1.0)
    ids = np.arange(4096, dtype=np.int32)
    p = ti.Pkm(c1, c2)
    p.register(cents, ids)
    addr, ad = p.query_host(q)
    ref = _oracle_assign(c1, c2, q)
    np.testing.assert_array_equal(addr, ref)
    np.testing.assert_array_equal(ad, _oracle_table(c1, c2, cents, ids)[ref])
    p.close()


def test_pkm_ties_and_collisions():
    c1 = oracle.fill_f32("t.c1", (64, 32), 1, 1.0)
    c2 = oracle.fill_f32("t.c2", (64, 32), 1, 1.0)
    c1[40] = c1[7]  # duplicated code words: the lower index wins
    c2[63] = c2[5]
    q = np.stack([np.concatenate([c1[7], c2[5]]), np.concatenate([c1[40], c2[63]]),
                  np.concatenate([c1[3], c2[60]])]).astype(np.float32)
    p = ti.Pkm(c1, c2)
    # three adapters on one address, one elsewhere: collisions keep the lowest id
    cents = np.stack([q[0], q[0], q[0], q[2]])
    p.register(cents, np.array([9, 4, 6, 2], np.int32))
    addr, ad = p.query_host(q)
    assert list(addr) == [7 * 64 + 5, 7 * 64 + 5, 3 * 64 + 60]
    assert list(ad) == [4, 4, 2]
    np.testing.assert_array_equal(addr, _oracle_assign(c1, c2, q))
    # an address nobody registered
    a2, d2 = p.query_host(np.concatenate([c1[1], c2[2]])[None])
    assert a2[0] == 1 * 64 + 2 and d2[0] == -1
    p.close()
