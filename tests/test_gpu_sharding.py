"""The table-sharded embedding layer on the GPU path (helrm_b200/sharding.py).

On one GPU the ranks are emulated in turn: each shard's transform, rescale,
fold, mask and rescale run through the C ABI on the same input ciphertexts,
the partial residues are summed as 64-bit integers in device memory (what
the NCCL reduce does across GPUs), and helrm_NewCiphertextsFromDeviceSum
imports the sum with every limb reduced modulo its prime.  Checked:

* the imported residues equal the host's modular sum of the partials;
* the merged ciphertext decrypts to the unsharded embedding within the
  north star's 2^-15 relative tolerance;
* one shard's partial ciphertext equals the oracle's run of the same steps
  (BSGS transform, rescale, fold rotations, mask product, rescale), residue
  for residue.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig
from helrm_b200 import sharding as S
from helrm_b200 import workload as W
from test_sharding_cpu import SMALL_VOCAB, small_case

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[40] + [36] * 5, logp=[60, 60], logscale=36, h=64)
REL_TOL = 2.0 ** -15


@pytest.fixture(scope="module")
def pair(oracle_mod):
    p = Pair(CFG, dnum=3, seed=20261215, oracle_mod=oracle_mod)
    yield p
    p.close()


def _inputs(pair, n, level):
    M, x0 = small_case()
    xs = [x0]
    for i in range(1, n):
        q = W.zipf_queries(SMALL_VOCAB, 1, seed=40 + i)[0]
        xs.append(W.selector(q, SMALL_VOCAB, 8))
    cts = []
    for x in xs:
        v = np.zeros(pair.slots)
        v[:len(x)] = x
        cts.append(pair.encrypt(v, level))
    return M, xs, cts


@pytest.mark.parametrize("nshards", [2, 3])
def test_sharded_merge_matches_unsharded(pair, nshards):
    import torch
    level = pair.info["max_level"]
    M, xs, cts = _inputs(pair, 2, level)
    nq_out = level - 1  # two rescales: the transform's and the mask's
    words = 2 * nq_out * pair.N
    total = torch.zeros((len(cts), words), dtype=torch.int64, device="cuda")
    host_sum = np.zeros((len(cts), 2, nq_out, pair.N), dtype=object)
    for tb in S.table_shards(len(SMALL_VOCAB), nshards):
        se = S.ShardedEmbedding(pair.lib, M, tb, level)
        outs = se.evaluate(cts)
        assert all(pair.lib.GetCiphertextLevel(o) == level - 2 for o in outs)
        part = torch.empty_like(total)
        pair.lib.CiphertextsToDevice(outs, part.data_ptr(), words)
        total += part
        for i, o in enumerate(outs):
            host_sum[i] += pair.ct_data(o).astype(object)
        scale = pair.lib.GetCiphertextScale(outs[0])
        for o in outs:
            pair.lib.DeleteCiphertext(o)
        se.close()
    torch.cuda.synchronize()  # the import orders only the library's own stream
    merged = pair.lib.NewCiphertextsFromDeviceSum(total.data_ptr(), len(cts), level - 2, 2, scale)
    qs = np.array(pair.o.primes[:nq_out], dtype=object)[None, :, None]
    for i, m in enumerate(merged):
        assert np.array_equal(pair.ct_data(m), (host_sum[i] % qs).astype(np.uint64))
        got = pair.decrypt(m)
        ref = M.astype(np.float64) @ xs[i]
        rows = M.shape[0]
        assert np.abs(got[:rows] - ref).max() <= REL_TOL * np.abs(ref).max()
        # slots of the unused rows of the layout period stay (near) zero
        period = S.layout_period(rows)
        assert np.abs(got[rows:period]).max() <= REL_TOL * np.abs(ref).max()


def test_shard_partial_bit_exact_vs_oracle(pair):
    level = pair.info["max_level"]
    M, xs, cts = _inputs(pair, 1, level)
    tb = S.table_shards(len(SMALL_VOCAB), 2)[1]
    se = S.ShardedEmbedding(pair.lib, M, tb, level)
    out = se.evaluate(cts)[0]
    o = pair.o
    plan = W.bsgs_plan(se.ks, se.ratio, pair.slots)
    gal = {o.galois(d) for d in plan["rotation_keys"]} | {o.galois(pair.slots >> i) for i in range(1, se.rot + 1)}
    keys = {g: pair.key(g) for g in gal}
    pts = [pair.lib.GetLinearTransformPlaintext(se.lt, k) for k in se.ks]
    y = o.pcmm(pair.ct_data(cts[0]), se.ks, pts, plan["stride"], keys, se.rot)
    y = o.rescale(o.mac([y], [pair.lib.GetPlaintextData(se.mask_pt)]))
    assert np.array_equal(pair.ct_data(out), y)
    se.close()
