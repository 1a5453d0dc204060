"""Table sharding of the embedding PCMM on CPU (helrm_b200/sharding.py).

* The layout algebra: every rank's masked, folded shard output, summed
  over the ranks, equals the unsharded transform's folded output on every
  slot (cleartext, the cfg2 matrix at LogN 16, 2 / 4 / 8 ranks).
* The exchange: world_size-2 gloo ranks each encrypt their shard's output
  under the shared key (the CPU oracle stands in for the GPU), sum the
  residues with one reduce and rank 0 reduces them modulo q.  The result is
  bit-exact against the single-process modular sum and decrypts to the
  unsharded embedding.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from helrm_b200 import sharding as S  # noqa: E402
from helrm_b200 import workload as W  # noqa: E402

# a small block-diagonal workload for the oracle runs (LogN 11: 1024 slots)
SMALL_VOCAB = [5, 40, 300, 9, 70, 1000]
SMALL_BASE = 8


def small_case():
    M = W.block_diag_matrix(SMALL_VOCAB, SMALL_BASE, 16, 0.05, seed=3)
    q = W.zipf_queries(SMALL_VOCAB, 1, seed=5)[0]
    x = W.selector(q, SMALL_VOCAB, SMALL_BASE)
    return M, x


def test_table_shards_balanced():
    assert [len(r) for r in S.table_shards(26, 8)] == [4, 4, 3, 3, 3, 3, 3, 3]
    assert [len(r) for r in S.table_shards(26, 4)] == [7, 7, 6, 6]
    assert [len(r) for r in S.table_shards(26, 1)] == [26]
    for n in (1, 2, 3, 8):
        parts = S.table_shards(26, n)
        assert sum(len(p) for p in parts) == 26 and parts[0].start == 0 and parts[-1].stop == 26
    with pytest.raises(ValueError):
        S.table_shards(3, 4)


def test_shard_matrix_block_height_and_rows():
    V = W.cfg2_vocab()
    M = W.block_diag_matrix(V, 64, 16, 0.05, seed=0)
    for n, bh in ((2, 256), (4, 128), (8, 64)):
        for tb in S.table_shards(26, n):
            Vm, h, R0, rows = S.shard_matrix(M, tb)
            assert h == bh and rows == 16 * len(tb) and R0 == 16 * tb.start
            for i in range(rows):
                assert np.array_equal(Vm[(R0 + i) % h], M[R0 + i])


@pytest.mark.parametrize("nshards", [2, 4, 8])
def test_masked_merge_equals_unsharded(nshards):
    V = W.cfg2_vocab()
    M = W.block_diag_matrix(V, 64, 16, 0.05, seed=0)
    slots = 32768
    x = W.selector(W.zipf_queries(V, 1)[0], V)
    d, rot = W.diagonalize(M, slots, "hybrid")
    xp = np.zeros(slots)
    xp[:len(x)] = x
    full = W.hybrid_fold(W.cleartext_lt(xp, d[(0, 0)], slots), slots, rot)
    merged = sum(S.cleartext_shard(M, tb, x, slots) for tb in S.table_shards(26, nshards))
    assert np.array_equal(merged, full)
    assert np.allclose(full[:416], M.astype(np.float64) @ x)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_rank(rank, world, port, out):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
                       "MASTER_PORT": str(port)})
    sys.path.insert(0, ROOT)
    import datetime

    import torch
    import torch.distributed as dist

    from oracle import oracle as om
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        M, x = small_case()
        main, aux = om.scheme_primes([36, 36, 36], [60], 11)
        o = om.Oracle(11, main, aux, 1)
        sk = o.secret_ntt(o.sample_secret(77, 32))  # the key every rank shares
        slots = o.N // 2
        tb = S.table_shards(len(SMALL_VOCAB), world)[rank]
        y = S.cleartext_shard(M, tb, x, slots)
        ct = o.encrypt(sk, o.encode(y, 3, 2.0 ** 30), 1000 + rank)
        buf = torch.from_numpy(ct.view(np.int64).copy())
        S.exchange_sum(buf, dist, dst=0)
        out.put((rank, ct, buf.numpy().copy() if rank == 0 else None))
    finally:
        dist.destroy_process_group()


def test_exchange_gloo_world2_bit_exact():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, ct, summed = q.get(timeout=180)
        res[rank] = (ct, summed)
    for p in procs:
        p.join(timeout=60)
    assert [p.exitcode for p in procs] == [0] * world
    from oracle import oracle as om
    main, aux = om.scheme_primes([36, 36, 36], [60], 11)
    o = om.Oracle(11, main, aux, 1)
    got = S.reduce_mod_q(res[0][1], main)
    qs = np.array(main, dtype=object)[None, :, None]
    want = ((res[0][0].astype(object) + res[1][0].astype(object)) % qs).astype(np.uint64)
    assert np.array_equal(got, want)  # the exchange is the single-process modular sum
    # and it decrypts to the unsharded embedding
    M, x = small_case()
    sk = o.secret_ntt(o.sample_secret(77, 32))
    dec = o.decode(o.decrypt(sk, got), 2.0 ** 30)
    rows = M.shape[0]
    assert np.abs(dec[:rows] - M.astype(np.float64) @ x).max() < 1e-5
